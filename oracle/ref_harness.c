/*
 * Test infrastructure only: a thin exporter around the reference's own CPU
 * KV-cache code.  It compiles the reference translation unit sf37.c
 * (found through -I$(REF_DIR)) with the reference Makefile flags and
 * re-exports the static functions the KV hot path is built from, so that the
 * oracle restatement and the CUDA library can be checked against the
 * reference's real arithmetic.  Nothing in the product links this file.
 *
 * Re-exported (reference file:line):
 *   kv_cache_push                      sf37.c:2054-2064
 *   attention_decode                   sf37.c:2066-2101
 *   gate loop after attention          sf37.c:2235-2239 (sf37_sigmoid, sf37_ops.c:9-16)
 *   payload_encode_kv_row_i8_grouped   sf37.c:6633-6659
 *   payload_decode_kv_row_i8_grouped   sf37.c:6661-6674
 *   payload_encoded_kv_row_bytes       sf37.c:6628-6631
 *   sf37_session_save_snapshot / _load_snapshot  sf37.c:7235-7500
 *   sf37_session_save_payload / _load_payload    sf37.c:6922-7233
 */
#include "sf37.c"

#include <pthread.h>
#include <unistd.h>

/* One linear CPU layer cache, as sf37_layer_kv_cache (sf37.c:199-204). */
uint64_t sf37ref_layer_cache_bytes(uint32_t cap) {
    return (uint64_t)cap * SF37_KV_HEADS * SF37_HEAD_DIM * sizeof(float);
}

/* Push n rows (k, v each [n][1024] f32) into a cache of capacity cap that
 * currently holds *n_live rows; on return *n_live is the new count. */
void sf37ref_kv_cache_push_rows(float *k_cache, float *v_cache, uint32_t cap,
                                uint32_t *n_live, const float *k, const float *v,
                                uint32_t n) {
    sf37_layer_kv_cache layer;
    layer.k = k_cache;
    layer.v = v_cache;
    layer.n = *n_live;
    layer.cap = cap;
    const uint64_t row = (uint64_t)SF37_KV_HEADS * SF37_HEAD_DIM;
    for (uint32_t i = 0; i < n; i++) kv_cache_push(&layer, k + i * row, v + i * row);
    *n_live = layer.n;
}

/* attention_decode + the sigmoid gate of run_layer_decode.  gate may be NULL
 * (no gating, as attention_decode alone). */
void sf37ref_attention_decode(float *out, const float *q, const float *k_cache,
                              const float *v_cache, uint32_t n_live, uint32_t cap,
                              uint32_t q_heads, int sliding, const float *gate) {
    sf37_layer_kv_cache layer;
    layer.k = (float *)k_cache;
    layer.v = (float *)v_cache;
    layer.n = n_live;
    layer.cap = cap;
    attention_decode(out, q, &layer, q_heads, sliding != 0);
    if (gate) {
        for (uint32_t h = 0; h < q_heads; h++) {
            const float g = sf37_sigmoid(gate[h]);
            float *head = out + (uint64_t)h * SF37_HEAD_DIM;
            for (uint32_t d = 0; d < SF37_HEAD_DIM; d++) head[d] *= g;
        }
    }
}

uint64_t sf37ref_payload_row_bytes(uint32_t elems, uint32_t group) {
    return payload_encoded_kv_row_bytes(elems, group);
}

void sf37ref_payload_encode_rows(const float *src, uint32_t elems, uint32_t group,
                                 uint64_t n_rows, uint8_t *dst) {
    const uint64_t eb = payload_encoded_kv_row_bytes(elems, group);
    for (uint64_t r = 0; r < n_rows; r++)
        payload_encode_kv_row_i8_grouped(src + r * elems, elems, group, dst + r * eb);
}

void sf37ref_payload_decode_rows(const uint8_t *src, uint32_t elems, uint32_t group,
                                 uint64_t n_rows, float *dst) {
    const uint64_t eb = payload_encoded_kv_row_bytes(elems, group);
    for (uint64_t r = 0; r < n_rows; r++)
        payload_decode_kv_row_i8_grouped(src + r * eb, elems, group, dst + r * elems);
}

/* ---- multi-threaded driver for the timed CPU baseline ----
 * The reference CPU path is single-threaded (one layer after another).  For
 * the CPU baseline the independent layers of the synthetic stack are spread
 * over worker threads; each layer still runs the reference's own
 * kv_cache_push + attention_decode + gate. */
typedef struct {
    float **k, **v, **q, **out, **gate, **k_new, **v_new;
    uint32_t *n_live, cap, q_heads;
    const int *sliding;
    uint32_t l0, l1;
} sf37ref_job;

static void *sf37ref_worker(void *arg) {
    sf37ref_job *j = (sf37ref_job *)arg;
    for (uint32_t l = j->l0; l < j->l1; l++) {
        sf37ref_kv_cache_push_rows(j->k[l], j->v[l], j->cap, &j->n_live[l],
                                   j->k_new[l], j->v_new[l], 1);
        sf37ref_attention_decode(j->out[l], j->q[l], j->k[l], j->v[l], j->n_live[l],
                                 j->cap, j->q_heads, j->sliding[l], j->gate[l]);
    }
    return NULL;
}

/* One decode step of n_layers independent layers on n_threads threads. */
int sf37ref_decode_step_layers(float **k, float **v, uint32_t *n_live, uint32_t cap,
                               float **k_new, float **v_new, float **q, float **gate,
                               float **out, const int *sliding, uint32_t q_heads,
                               uint32_t n_layers, uint32_t n_threads) {
    if (n_threads == 0) n_threads = 1;
    if (n_threads > n_layers) n_threads = n_layers;
    pthread_t th[256];
    sf37ref_job jobs[256];
    if (n_threads > 256) n_threads = 256;
    uint32_t per = (n_layers + n_threads - 1) / n_threads;
    uint32_t started = 0;
    for (uint32_t t = 0; t < n_threads; t++) {
        sf37ref_job *j = &jobs[t];
        j->k = k; j->v = v; j->q = q; j->out = out; j->gate = gate;
        j->k_new = k_new; j->v_new = v_new; j->n_live = n_live; j->cap = cap;
        j->q_heads = q_heads; j->sliding = sliding;
        j->l0 = t * per;
        j->l1 = j->l0 + per > n_layers ? n_layers : j->l0 + per;
        if (j->l0 >= j->l1) break;
        if (pthread_create(&th[t], NULL, sf37ref_worker, j) != 0) return 0;
        started++;
    }
    for (uint32_t t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 1;
}

/* ---- session checkpoints through the reference's own writers/loaders ----
 * A CPU-backend sf37_session (no engine, sf37.c:4510-4533) is filled with
 * the given state and handed to sf37_session_save_snapshot (sf37.c:7235),
 * sf37_session_save_payload (6922), sf37_session_load_snapshot (7347) or
 * sf37_session_load_payload (7038).  On the CPU backend a layer's live rows
 * are layer->k / layer->v rows [n - rows, n) (sf37.c:7322-7336), and the raw
 * snapshot stores a layer's K rows followed by its V rows; the payload rows
 * are K, V interleaved as on the CUDA backend. */
static void sf37ref_session_init(sf37_session *s, int ctx, const int *tokens, int n_tokens,
                                 float *logits, float *hidden, float **k, float **v,
                                 const uint32_t *n_rows) {
    memset(s, 0, sizeof(*s));
    s->ctx_size = ctx;
    s->checkpoint.v = (int *)malloc(sizeof(int) * (size_t)(n_tokens > 0 ? n_tokens : 1));
    if (n_tokens > 0) memcpy(s->checkpoint.v, tokens, sizeof(int) * (size_t)n_tokens);
    s->checkpoint.len = n_tokens;
    s->checkpoint.cap = n_tokens > 0 ? n_tokens : 1;
    s->checkpoint_valid = true;
    s->logits = logits;
    s->hidden = hidden;
    for (uint32_t il = 0; il < SF37_MAIN_LAYERS; il++) {
        s->cpu_cache.layer[il].k = k[il];
        s->cpu_cache.layer[il].v = v[il];
        s->cpu_cache.layer[il].n = n_rows ? n_rows[il] : 0;
        s->cpu_cache.layer[il].cap = (uint32_t)ctx;
    }
    s->cpu_cache.cap = (uint32_t)ctx;
}

/* kind 0: raw snapshot, 1: payload.  Returns the bytes written into out,
 * or -1 with the reference's message in err. */
int64_t sf37ref_session_save(int kind, int ctx, const int *tokens, int n_tokens, float *logits,
                             float *hidden, float **k, float **v, const uint32_t *n_rows,
                             uint8_t *out, uint64_t out_cap, char *err, size_t errlen) {
    sf37_session s;
    sf37ref_session_init(&s, ctx, tokens, n_tokens, logits, hidden, k, v, n_rows);
    int64_t n = -1;
    if (kind == 0) {
        sf37_session_snapshot snap = {0};
        if (sf37_session_save_snapshot(&s, &snap, err, errlen) == 0 && snap.len <= out_cap) {
            memcpy(out, snap.ptr, (size_t)snap.len);
            n = (int64_t)snap.len;
        }
        sf37_session_snapshot_free(&snap);
    } else {
        FILE *fp = tmpfile();
        if (fp && sf37_session_save_payload(&s, fp, err, errlen) == 0) {
            const long len = ftell(fp);
            rewind(fp);
            if (len >= 0 && (uint64_t)len <= out_cap && fread(out, 1, (size_t)len, fp) == (size_t)len)
                n = len;
        }
        if (fp) fclose(fp);
    }
    free(s.checkpoint.v);
    return n;
}

/* Loads buf into a CPU session of context ctx whose layer caches k[il],
 * v[il] hold ctx rows each.  Returns the reference's code (0 = success);
 * on success n_rows[il] = the rows restored, tokens / *n_tokens / logits /
 * hidden are written. */
int sf37ref_session_load(int kind, const uint8_t *buf, uint64_t len, int ctx, int *tokens,
                         int *n_tokens, float *logits, float *hidden, float **k, float **v,
                         uint32_t *n_rows, char *err, size_t errlen) {
    sf37_session s;
    sf37ref_session_init(&s, ctx, NULL, 0, logits, hidden, k, v, NULL);
    int rc;
    if (kind == 0) {
        sf37_session_snapshot snap = {(uint8_t *)buf, len, len};
        rc = sf37_session_load_snapshot(&s, &snap, err, errlen);
    } else {
        FILE *fp = tmpfile();
        rc = 1;
        if (fp && fwrite(buf, 1, (size_t)len, fp) == (size_t)len) {
            rewind(fp);
            rc = sf37_session_load_payload(&s, fp, len, err, errlen);
        }
        if (fp) fclose(fp);
    }
    if (rc == 0) {
        *n_tokens = s.checkpoint.len;
        if (s.checkpoint.len > 0) memcpy(tokens, s.checkpoint.v, sizeof(int) * (size_t)s.checkpoint.len);
        for (uint32_t il = 0; il < SF37_MAIN_LAYERS; il++) n_rows[il] = s.cpu_cache.layer[il].n;
    }
    free(s.checkpoint.v);
    return rc;
}

/* ---- the reference's CUDA-backend per-row checkpoint loops (timing) ----
 * The session writers read each live row with two synchronous 4 KiB
 * sf37_cuda_tensor_read calls (sf37.c:7298-7320 snapshot, 6976-7009
 * payload).  These restate those loops for one layer with the reference's
 * own tensor_read (passed in from the reference CUDA library) and encoder,
 * so the bench can time the reference path on a B200.  Rows are f32
 * [cap][1024]. */
typedef int (*sf37ref_read_fn)(const void *tensor, uint64_t off, void *dst, uint64_t bytes);

int sf37ref_snapshot_rows_cuda(sf37ref_read_fn rd, const void *k_tensor, const void *v_tensor,
                               uint32_t first_pos, uint32_t rows, uint32_t cap, uint8_t *dst) {
    const uint64_t row = (uint64_t)SF37_KV_HEADS * SF37_HEAD_DIM * sizeof(float);
    for (uint32_t r = 0; r < rows; r++) {
        const uint64_t off = (uint64_t)((first_pos + r) % cap) * row;
        if (!rd(k_tensor, off, dst, row)) return 1;
        dst += row;
        if (!rd(v_tensor, off, dst, row)) return 1;
        dst += row;
    }
    return 0;
}

int sf37ref_payload_rows_cuda(sf37ref_read_fn rd, const void *k_tensor, const void *v_tensor,
                              uint32_t first_pos, uint32_t rows, uint32_t cap, int fd) {
    const uint32_t kv_row = SF37_KV_HEADS * SF37_HEAD_DIM;
    const uint32_t group = SF37_SESSION_PAYLOAD_KV_GROUP;
    const uint64_t enc_bytes = payload_encoded_kv_row_bytes(kv_row, group);
    float row_buf[SF37_KV_HEADS * SF37_HEAD_DIM];
    uint8_t enc[SF37_KV_HEADS * SF37_HEAD_DIM + 64 * sizeof(float)];
    FILE *fp = fdopen(dup(fd), "wb");
    if (!fp) return 1;
    int rc = 0;
    for (uint32_t r = 0; rc == 0 && r < rows; r++) {
        const uint64_t off = (uint64_t)((first_pos + r) % cap) * kv_row * sizeof(float);
        for (int which = 0; which < 2 && rc == 0; which++) {
            if (!rd(which ? v_tensor : k_tensor, off, row_buf, (uint64_t)kv_row * sizeof(float))) rc = 1;
            else {
                payload_encode_kv_row_i8_grouped(row_buf, kv_row, group, enc);
                if (fwrite(enc, 1, (size_t)enc_bytes, fp) != (size_t)enc_bytes) rc = 1;
            }
        }
    }
    if (fclose(fp) != 0) rc = 1;
    return rc;
}

/* ---- q/k head preparation, the reference CPU form ----
 * head_rms_norm_weight1 (sf37.c:1921) + apply_rope_one (sf37.c:2015) on
 * n_head heads of x in place; w: f32 [128] (the bf16 weights widened, as
 * tensor_bf16_to_f32 does, sf37.c:2223). */
void sf37ref_qk_prep(float *x, uint32_t n_head, const float *w, uint32_t rotary_dim, double theta,
                     int llama3, uint32_t pos) {
    head_rms_norm_weight1(x, n_head, SF37_HEAD_DIM, w, SF37_RMS_EPS);
    apply_rope_one(x, n_head, SF37_HEAD_DIM, rotary_dim, theta, llama3 != 0, pos);
}

/* ---- sf37_kvstore records through the reference's own store path ----
 * sf37_kvstore_store_live_prefix_text (sf37_kvstore.c:929-1158) on a
 * CPU-backend session, with the text given (cache_text_override), into a
 * kvstore opened on `dir` (min_tokens 1).  The record lands in
 * dir/<sha1(text)>.kv.  Returns 1 when the reference stored it. */
#include "sf37_kvstore.h"

int sf37ref_kvstore_store(const char *dir, int ctx, const int *tokens, int n_tokens, float *logits,
                          float *hidden, float **k, float **v, const uint32_t *n_rows, const char *text,
                          char *err, size_t errlen) {
    sf37_session s;
    sf37ref_session_init(&s, ctx, tokens, n_tokens, logits, hidden, k, v, n_rows);
    sf37_kvstore kc;
    sf37_kvstore_options opt = sf37_kvstore_default_options();
    opt.min_tokens = 1;
    int ok = 0;
    if (sf37_kvstore_open(&kc, dir, 1u << 20, false, opt, "ref", NULL, NULL)) {
        sf37_tokens tk = {0};
        for (int i = 0; i < n_tokens; i++) sf37_tokens_push(&tk, tokens[i]);
        ok = sf37_kvstore_store_live_prefix_text(&kc, NULL, &s, &tk, n_tokens, "cold", text, 0, NULL, NULL, err,
                                                 errlen) ? 1 : 0;
        sf37_tokens_free(&tk);
        sf37_kvstore_close(&kc);
    }
    free(s.checkpoint.v);
    return ok;
}

void sf37ref_kvstore_fill_header(uint8_t *h, uint8_t model_id, uint8_t quant_bits, uint8_t reason,
                                 uint8_t ext_flags, uint32_t tokens, uint32_t hits, uint32_t ctx_size,
                                 uint64_t created_at, uint64_t last_used, uint64_t payload_bytes) {
    sf37_kvstore_fill_header(h, model_id, quant_bits, reason, ext_flags, tokens, hits, ctx_size, created_at,
                             last_used, payload_bytes);
}

void sf37ref_sha1_hex(const void *p, size_t n, char out[41]) { sf37_kvstore_sha1_bytes_hex(p, n, out); }
