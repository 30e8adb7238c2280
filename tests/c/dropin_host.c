/*
 * A C host using libsf37kv the way sf37.c uses the reference's CUDA backend
 * for one decode layer (sf37.c:3356-3366): tensor handles, the ring append,
 * the decode at a position, and a raw/payload session record round trip
 * through the sf37kv_session C API.  Checks against a naive double-precision
 * attention computed here.  Exit status 0 = every check passed.
 */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "sf37_cuda_kv.h"
#include "sf37kv.h"
#include "sf37kv_session.h"

enum { QH = 64, KVH = 8, HD = 128, KV = KVH * HD, CAP = 600, POS = 700 };

static uint64_t rng = 0x9E3779B97F4A7C15ull;
static float frand(void) {
    rng ^= rng << 13;
    rng ^= rng >> 7;
    rng ^= rng << 17;
    return (float)((double)(rng >> 11) / 9007199254740992.0 * 2.0 - 1.0);
}

static int fail(const char *what) {
    fprintf(stderr, "FAIL: %s (%s)\n", what, sf37kv_last_error());
    return 1;
}

int main(void) {
    if (!sf37_cuda_init()) return fail("init");
    float *k = malloc(sizeof(float) * CAP * KV), *v = malloc(sizeof(float) * CAP * KV);
    float q[QH * HD], gate[QH], kn[KV], vn[KV], out[QH * HD];
    for (int i = 0; i < CAP * KV; i++) {
        k[i] = frand();
        v[i] = frand();
    }
    for (int i = 0; i < QH * HD; i++) q[i] = frand();
    for (int i = 0; i < QH; i++) gate[i] = frand();
    for (int i = 0; i < KV; i++) {
        kn[i] = frand();
        vn[i] = frand();
    }
    sf37_cuda_tensor *tk = sf37_cuda_tensor_alloc((uint64_t)CAP * KV * 4), *tv = sf37_cuda_tensor_alloc((uint64_t)CAP * KV * 4);
    sf37_cuda_tensor *tq = sf37_cuda_tensor_alloc(sizeof(q)), *tg = sf37_cuda_tensor_alloc(sizeof(gate));
    sf37_cuda_tensor *tkn = sf37_cuda_tensor_alloc(sizeof(kn)), *tvn = sf37_cuda_tensor_alloc(sizeof(vn));
    sf37_cuda_tensor *to = sf37_cuda_tensor_alloc(sizeof(out));
    if (!tk || !tv || !tq || !tg || !tkn || !tvn || !to) return fail("alloc");
    if (!sf37_cuda_tensor_write(tk, 0, k, (uint64_t)CAP * KV * 4) || !sf37_cuda_tensor_write(tv, 0, v, (uint64_t)CAP * KV * 4) ||
        !sf37_cuda_tensor_write(tq, 0, q, sizeof(q)) || !sf37_cuda_tensor_write(tg, 0, gate, sizeof(gate)) ||
        !sf37_cuda_tensor_write(tkn, 0, kn, sizeof(kn)) || !sf37_cuda_tensor_write(tvn, 0, vn, sizeof(vn)))
        return fail("write");
    /* the engine's step: store the new row at POS (ring slot POS % CAP), then attend at POS */
    if (!sf37_cuda_store_kv_cache_batch(tk, tv, tkn, tvn, POS, 1, CAP, KV)) return fail("store");
    if (!sf37_cuda_attention_decode_heads_at(to, tq, tk, tv, tg, POS, CAP, QH, KVH, HD, 1, 512)) return fail("decode");
    if (!sf37_cuda_tensor_read(to, 0, out, sizeof(out))) return fail("read");
    memcpy(k + (POS % CAP) * KV, kn, sizeof(kn));
    memcpy(v + (POS % CAP) * KV, vn, sizeof(vn));
    /* naive reference: sliding window 512 ending at POS */
    double worst = 0;
    for (int h = 0; h < QH; h++) {
        const int g = h / (QH / KVH);
        double m = -1e300, l = 0, acc[HD] = {0};
        for (int p = POS - 511; p <= POS; p++) {
            const float *kr = k + (p % CAP) * KV + g * HD;
            double s = 0;
            for (int d = 0; d < HD; d++) s += (double)q[h * HD + d] * kr[d];
            s /= sqrt((double)HD);
            if (s > m) {
                const double a = exp(m - s);
                l *= a;
                for (int d = 0; d < HD; d++) acc[d] *= a;
                m = s;
            }
            const double e = exp(s - m);
            l += e;
            const float *vr = v + (p % CAP) * KV + g * HD;
            for (int d = 0; d < HD; d++) acc[d] += e * vr[d];
        }
        const double sg = 1.0 / (1.0 + exp(-(double)gate[h]));
        for (int d = 0; d < HD; d++) {
            const double want = acc[d] / l * sg, got = out[h * HD + d];
            const double err = fabs(got - want);
            if (err > 6e-5 && err > 1e-4 * fabs(want)) {
                fprintf(stderr, "FAIL: head %d dim %d got %g want %g\n", h, d, got, want);
                return 1;
            }
            if (err > worst) worst = err;
        }
    }

    /* session records over the same cache as a 1-layer layout */
    sf37kv_session_layout L = sf37kv_session_layout_default();
    L.n_layers = 1;
    L.vocab = 16;
    L.embd = 8;
    L.full_every = 0; /* the one layer is a sliding ring of 600 slots, not a full layer */
    sf37kv_cache cache = {tk->ptr, tv->ptr, CAP, 1, 512, 0};
    int32_t toks[POS + 1];
    for (int i = 0; i <= POS; i++) toks[i] = i % 16;
    float logits[16] = {0}, hidden[8] = {0};
    sf37kv_session s = {L, 1024, POS + 1, toks, logits, hidden, &cache, SF37KV_F32, 1};
    char err[256];
    const uint64_t snap_bytes = sf37kv_session_snapshot_bytes(&s);
    void *snap = sf37kv_host_alloc(snap_bytes);
    uint64_t len = 0;
    if (!snap || sf37kv_session_save_snapshot(&s, snap, snap_bytes, &len, err, sizeof(err)) || len != snap_bytes)
        return fail("save_snapshot");
    char path[] = "/tmp/sf37kv_payloadXXXXXX";
    const int fd = mkstemp(path);
    if (fd < 0) return fail("mkstemp");
    unlink(path);
    if (sf37kv_session_save_payload(&s, fd, err, sizeof(err))) return fail(err);
    const uint64_t pay_bytes = sf37kv_session_payload_bytes(&s);
    if ((uint64_t)lseek(fd, 0, SEEK_CUR) != pay_bytes) return fail("payload size");
    /* restore the snapshot into a cleared cache and compare the live rows */
    float *zero = calloc((size_t)CAP * KV, 4);
    sf37_cuda_tensor_write(tk, 0, zero, (uint64_t)CAP * KV * 4);
    s.n_tokens = 0;
    if (sf37kv_session_load_snapshot(&s, snap, len, err, sizeof(err))) return fail(err);
    float *back = malloc(sizeof(float) * CAP * KV);
    sf37_cuda_tensor_read(tk, 0, back, (uint64_t)CAP * KV * 4);
    for (int p = POS + 1 - CAP; p <= POS; p++)
        if (memcmp(back + (p % CAP) * KV, k + (p % CAP) * KV, KV * 4)) return fail("snapshot row");
    lseek(fd, 0, SEEK_SET);
    if (sf37kv_session_load_payload(&s, fd, pay_bytes, err, sizeof(err)) || s.n_tokens != POS + 1)
        return fail("load_payload");
    close(fd);
    printf("OK: decode max err %.3g; snapshot %llu B, payload %llu B\n", worst, (unsigned long long)snap_bytes,
           (unsigned long long)pay_bytes);
    sf37kv_host_free(snap);
    free(zero);
    free(back);
    free(k);
    free(v);
    sf37_cuda_tensor *all[] = {tk, tv, tq, tg, tkn, tvn, to};
    for (int i = 0; i < 7; i++) sf37_cuda_tensor_free(all[i]);
    sf37_cuda_cleanup();
    return 0;
}
