/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of the reference's KV-cache hot-path arithmetic, used
 * by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker.  The shipped library (sf37_b200/libsf37kv.so) never calls it.
 *
 * Parity of this restatement is pinned against the reference's own code
 * compiled from its sources (oracle/_ref/libsf37ref.so, see ref_harness.c)
 * and against the committed fixtures under tests/golden/.
 *
 * Every function cites the reference it restates.  Caches are row-major
 * [cap][kv_heads][head_dim]; a "row" is one position (kv_heads*head_dim
 * elements).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------- f16 helpers ----------------
 * f16 -> f32 is exact (restates sf37_f16_to_f32, sf37_quant.c:5-31).
 * f32 -> f16 is IEEE-754 round-to-nearest-even with subnormals and inf/NaN.
 * The reference has no product f32->f16 KV conversion (its only converter,
 * tests/test_sf37_cuda_ops.cu:32-43, truncates and flushes subnormals), so
 * this is the conversion the f16 cache mode defines. */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 0) {
        if (m == 0) bits = sign;
        else {  /* subnormal: value = m * 2^-24 */
            float f = (float)m * (1.0f / 16777216.0f);
            memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (e == 31) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
    int32_t e = (int32_t)(ax >> 23) - 127;
    if (e >= -14) { /* normal f16 range */
        uint32_t mant = ax & 0x7fffffu;
        uint32_t hb = ((uint32_t)(e + 15) << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (hb & 1u))) hb++; /* may carry into exponent: fine */
        return (uint16_t)(sign | hb);
    }
    if (e < -25) return (uint16_t)sign; /* below half of the smallest subnormal */
    /* subnormal: value / 2^-24, rounded to nearest even */
    uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
    int shift = -e - 14 + 13;  /* 14..24 */
    uint32_t hb = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hb & 1u))) hb++;
    return (uint16_t)(sign | hb);
}

void orc_f32_to_f16_array(const float *src, uint16_t *dst, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) dst[i] = orc_f32_to_f16(src[i]);
}

void orc_f16_to_f32_array(const uint16_t *src, float *dst, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) dst[i] = orc_f16_to_f32(src[i]);
}

/* ---------------- append ----------------
 * Restates store_kv_cache_batch_kernel (sf37_cuda.cu:6355-6372): token t of
 * the batch lands in ring slot (pos0 + t) % cap.  elem_bytes 4 copies f32,
 * elem_bytes 2 converts f32 -> f16 (RNE). */
void orc_store_kv_rows(void *k_cache, void *v_cache, const float *k, const float *v,
                       uint32_t pos0, uint32_t n_tok, uint32_t cap, uint32_t kv_dim,
                       int elem_bytes) {
    for (uint32_t t = 0; t < n_tok; t++) {
        uint64_t slot = (uint64_t)((pos0 + t) % cap);
        for (uint32_t d = 0; d < kv_dim; d++) {
            uint64_t dst = slot * kv_dim + d, src = (uint64_t)t * kv_dim + d;
            if (elem_bytes == 4) {
                ((float *)k_cache)[dst] = k[src];
                ((float *)v_cache)[dst] = v[src];
            } else {
                ((uint16_t *)k_cache)[dst] = orc_f32_to_f16(k[src]);
                ((uint16_t *)v_cache)[dst] = orc_f32_to_f16(v[src]);
            }
        }
    }
}

/* ---------------- attention ----------------
 * sigmoid restates sf37_sigmoid (sf37_ops.c:9-16). */
static float orc_sigmoid(float x) {
    if (x >= 0.0f) {
        float z = expf(-x);
        return 1.0f / (1.0f + z);
    }
    float z = expf(x);
    return z / (1.0f + z);
}

/* Live-row window of one query at position pos (the causal "_at" form):
 * restates sf37_cuda.cu:2752-2758 / 3194-3199 and cpu_attention_prefill_ref
 * (tests/test_sf37_cuda_ops.cu:868-870): have = pos+1; rows older than cap
 * were overwritten; a sliding layer also drops rows older than window. */
static uint32_t orc_start_at(uint32_t pos, uint32_t cap, int sliding, uint32_t window) {
    uint32_t have = pos + 1u, start = 0;
    if (have > cap) start = have - cap;
    if (sliding && have > window && have - window > start) start = have - window;
    return start;
}

/* One head, rows [start, end) of logical positions, ring slot r % cap.
 * Two passes (max, then exp-sum) in f32, as attention_decode (sf37.c:
 * 2066-2101) and cpu_attention_decode (tests/test_sf37_cuda_ops.cu:208-250).
 * Output = acc / denom * sigmoid(gate); a zero denominator gives 0. */
static void orc_head(float *oh, const float *qh, const float *k_cache, const float *v_cache,
                     uint32_t start, uint32_t end, uint32_t cap, uint32_t kv_heads,
                     uint32_t kvh, uint32_t head_dim, const float *gate_h) {
    const uint64_t kv_row = (uint64_t)kv_heads * head_dim;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float max_score = -INFINITY;
    for (uint32_t r = start; r < end; r++) {
        const float *kh = k_cache + (uint64_t)(r % cap) * kv_row + (uint64_t)kvh * head_dim;
        float s = 0.0f;
        for (uint32_t d = 0; d < head_dim; d++) s += qh[d] * kh[d];
        s *= scale;
        if (s > max_score) max_score = s;
    }
    float *acc = (float *)calloc(head_dim, sizeof(float));
    float denom = 0.0f;
    for (uint32_t r = start; r < end; r++) {
        const uint64_t row = (uint64_t)(r % cap) * kv_row + (uint64_t)kvh * head_dim;
        const float *kh = k_cache + row, *vh = v_cache + row;
        float s = 0.0f;
        for (uint32_t d = 0; d < head_dim; d++) s += qh[d] * kh[d];
        s *= scale;
        float w = expf(s - max_score);
        denom += w;
        for (uint32_t d = 0; d < head_dim; d++) acc[d] += w * vh[d];
    }
    const float inv = denom > 0.0f ? 1.0f / denom : 0.0f;
    const float g = gate_h ? orc_sigmoid(*gate_h) : 1.0f;
    for (uint32_t d = 0; d < head_dim; d++) oh[d] = acc[d] * inv * g;
    free(acc);
}

/* sf37_cuda_attention_decode_heads_at semantics (sf37_cuda.cu:3079-3161):
 * one query at position pos over a ring cache of capacity cap. */
void orc_attention_decode_at(float *out, const float *q, const float *k_cache,
                             const float *v_cache, const float *gate, uint32_t pos,
                             uint32_t cap, uint32_t q_heads, uint32_t kv_heads,
                             uint32_t head_dim, int sliding, uint32_t window) {
    const uint32_t repeat = q_heads / kv_heads;
    const uint32_t start = orc_start_at(pos, cap, sliding, window);
    for (uint32_t h = 0; h < q_heads; h++)
        orc_head(out + (uint64_t)h * head_dim, q + (uint64_t)h * head_dim, k_cache, v_cache,
                 start, pos + 1u, cap, kv_heads, h / repeat, head_dim, gate ? gate + h : NULL);
}

/* sf37_cuda_attention_decode_heads semantics (sf37_cuda.cu:3003-3077 and
 * attention_decode_heads_kernel 2408-2457): n_cache live positions
 * 0..n_cache-1, sliding keeps the last window of them, no cap clamp. */
void orc_attention_decode_n(float *out, const float *q, const float *k_cache,
                            const float *v_cache, const float *gate, uint32_t n_cache,
                            uint32_t cap, uint32_t q_heads, uint32_t kv_heads,
                            uint32_t head_dim, int sliding, uint32_t window) {
    const uint32_t repeat = q_heads / kv_heads;
    uint32_t start = 0;
    if (sliding && n_cache > window) start = n_cache - window;
    for (uint32_t h = 0; h < q_heads; h++)
        orc_head(out + (uint64_t)h * head_dim, q + (uint64_t)h * head_dim, k_cache, v_cache,
                 start, n_cache, cap, kv_heads, h / repeat, head_dim, gate ? gate + h : NULL);
}

/* sf37_cuda_attention_prefill_heads semantics (sf37_cuda.cu:3241-3317,
 * cpu_attention_prefill_ref tests/test_sf37_cuda_ops.cu:859-905): token t of
 * the chunk is a query at pos0 + t; q [n_tok][q_heads][hd], gate [n_tok][q_heads].
 * Only tokens in [t0, t1) are computed (sampled checks at large sizes). */
void orc_attention_prefill(float *out, const float *q, const float *k_cache,
                           const float *v_cache, const float *gate, uint32_t pos0,
                           uint32_t n_tok, uint32_t cap, uint32_t q_heads, uint32_t kv_heads,
                           uint32_t head_dim, int sliding, uint32_t window,
                           uint32_t t0, uint32_t t1) {
    const uint64_t q_dim = (uint64_t)q_heads * head_dim;
    if (t1 > n_tok) t1 = n_tok;
    for (uint32_t t = t0; t < t1; t++)
        orc_attention_decode_at(out + t * q_dim, q + t * q_dim, k_cache, v_cache,
                                gate ? gate + (uint64_t)t * q_heads : NULL, pos0 + t, cap,
                                q_heads, kv_heads, head_dim, sliding, window);
}

/* ---------------- int8-grouped payload codec ----------------
 * Restates payload_encode/decode_kv_row_i8_grouped (sf37.c:6623-6674): per
 * group of `group` elements, scale = max|x| / 127 (1 if the group is all
 * zero), q = clamp(lrint(x / scale), -127, 127); encoded row = all group
 * scales (f32) then all int8 values.  Non-finite inputs are ignored for the
 * max and encoded as 0.
 *
 * variant 0: the source-literal IEEE arithmetic (scale = m / 127, x / scale).
 * variant 1: the arithmetic the reference executes when built with its own
 *   flags (-O3 -ffast-math, Makefile:11): the division by 127 becomes a
 *   multiply by the rounded constant 1/127, and x / scale becomes
 *   x * (1 / scale) with the reciprocal computed once per group:
 *   scale = m * (1/127), q = rint(x * (1/scale)).  Checked against the
 *   compiled reference in tests. */
uint64_t orc_payload_row_bytes(uint32_t elems, uint32_t group) {
    uint32_t groups = (elems + group - 1u) / group;
    return (uint64_t)groups * 4u + elems;
}

void orc_payload_encode_row(const float *src, uint32_t elems, uint32_t group, int variant,
                            uint8_t *dst) {
    uint32_t groups = (elems + group - 1u) / group;
    int8_t *qv = (int8_t *)(dst + (uint64_t)groups * 4u);
    for (uint32_t g = 0; g < groups; g++) {
        uint32_t b = g * group, e = b + group < elems ? b + group : elems;
        float m = 0.0f;
        for (uint32_t i = b; i < e; i++) {
            float a = fabsf(src[i]);
            if (isfinite(a) && a > m) m = a;
        }
        float scale, inv = 0.0f;
        if (m > 0.0f) {
            if (variant == 1) {
                scale = m * (1.0f / 127.0f);
                inv = 1.0f / scale;
            } else scale = m / 127.0f;
        } else {
            scale = 1.0f;
            inv = 1.0f;
        }
        memcpy(dst + (uint64_t)g * 4u, &scale, 4);
        for (uint32_t i = b; i < e; i++) {
            float x = src[i];
            if (!isfinite(x)) x = 0.0f;
            float y = variant == 1 ? x * inv : x / scale;
            long qi = lrintf(y);
            if (qi > 127) qi = 127;
            if (qi < -127) qi = -127;
            qv[i] = (int8_t)qi;
        }
    }
}

void orc_payload_decode_row(const uint8_t *src, uint32_t elems, uint32_t group, float *dst) {
    uint32_t groups = (elems + group - 1u) / group;
    const int8_t *qv = (const int8_t *)(src + (uint64_t)groups * 4u);
    for (uint32_t g = 0; g < groups; g++) {
        float scale;
        memcpy(&scale, src + (uint64_t)g * 4u, 4);
        uint32_t b = g * group, e = b + group < elems ? b + group : elems;
        for (uint32_t i = b; i < e; i++) dst[i] = (float)qv[i] * scale;
    }
}

/* ---------------- snapshot KV sections ----------------
 * The per-layer KV section of the CUDA-backend snapshots (raw:
 * sf37.c:7298-7320; payload: sf37.c:6980-7010): for r in 0..rows-1, physical
 * slot (first_pos + r) % cap, write the K row then the V row.  Raw rows are
 * f32 (kv_dim*4 bytes); payload rows are int8-grouped encoded.
 * elem_bytes selects an f32 (4) or f16 (2) cache; f16 is upcast exactly. */
static void orc_row_f32(const void *cache, int elem_bytes, uint64_t slot, uint32_t kv_dim,
                        float *row) {
    if (elem_bytes == 4) memcpy(row, (const float *)cache + slot * kv_dim, (size_t)kv_dim * 4);
    else
        for (uint32_t d = 0; d < kv_dim; d++)
            row[d] = orc_f16_to_f32(((const uint16_t *)cache)[slot * kv_dim + d]);
}

void orc_pack_layer(uint8_t *dst, const void *k_cache, const void *v_cache, int elem_bytes,
                    uint32_t first_pos, uint32_t rows, uint32_t cap, uint32_t kv_dim,
                    int fmt /*0 raw f32, 1 payload i8g*/, uint32_t group, int variant) {
    float *row = (float *)malloc((size_t)kv_dim * 4);
    uint64_t rb = fmt == 0 ? (uint64_t)kv_dim * 4u : orc_payload_row_bytes(kv_dim, group);
    for (uint32_t r = 0; r < rows; r++) {
        uint64_t slot = (uint64_t)((first_pos + r) % cap);
        for (int kv = 0; kv < 2; kv++) {
            orc_row_f32(kv == 0 ? k_cache : v_cache, elem_bytes, slot, kv_dim, row);
            uint8_t *o = dst + ((uint64_t)r * 2u + (uint64_t)kv) * rb;
            if (fmt == 0) memcpy(o, row, (size_t)kv_dim * 4);
            else orc_payload_encode_row(row, kv_dim, group, variant, o);
        }
    }
    free(row);
}

/* Restore (sf37.c:7410-7432 raw, 7146-7185 payload): the inverse scatter.
 * Into an f16 cache the decoded f32 value is converted with RNE. */
void orc_unpack_layer(const uint8_t *src, void *k_cache, void *v_cache, int elem_bytes,
                      uint32_t first_pos, uint32_t rows, uint32_t cap, uint32_t kv_dim,
                      int fmt, uint32_t group) {
    float *row = (float *)malloc((size_t)kv_dim * 4);
    uint64_t rb = fmt == 0 ? (uint64_t)kv_dim * 4u : orc_payload_row_bytes(kv_dim, group);
    for (uint32_t r = 0; r < rows; r++) {
        uint64_t slot = (uint64_t)((first_pos + r) % cap);
        for (int kv = 0; kv < 2; kv++) {
            const uint8_t *s = src + ((uint64_t)r * 2u + (uint64_t)kv) * rb;
            if (fmt == 0) memcpy(row, s, (size_t)kv_dim * 4);
            else orc_payload_decode_row(s, kv_dim, group, row);
            void *cache = kv == 0 ? k_cache : v_cache;
            if (elem_bytes == 4) memcpy((float *)cache + slot * kv_dim, row, (size_t)kv_dim * 4);
            else
                for (uint32_t d = 0; d < kv_dim; d++)
                    ((uint16_t *)cache)[slot * kv_dim + d] = orc_f32_to_f16(row[d]);
        }
    }
    free(row);
}

/* ---- q/k head preparation (the step before the append) ----
 * head_rms_norm_weight1 (sf37.c:1921-1929) with sf37_rms_norm_weight1
 * (sf37_ops.c:22-28) and apply_rope_one (sf37.c:2015-2031) with
 * sf37_inv_freq (sf37.c:1995-2013), on n_head heads of x in place.
 * w: bf16 bits [head_dim] (the model's q_norm / k_norm). */
static double orc_inv_freq(uint32_t pair, uint32_t dim, double theta, int llama3) {
    double inv = 1.0 / pow(theta, (double)(pair * 2u) / (double)dim);
    if (!llama3) return inv;
    const double factor = 2.0, low_ff = 1.0, high_ff = 32.0, old_ctx = 131072.0;
    const double low_wl = old_ctx / low_ff, high_wl = old_ctx / high_ff;
    const double wavelen = 2.0 * 3.14159265358979323846 / inv;
    if (wavelen > low_wl) return inv / factor;
    if (wavelen < high_wl) return inv;
    const double smooth = (old_ctx / wavelen - low_ff) / (high_ff - low_ff);
    return (1.0 - smooth) * inv / factor + smooth * inv;
}

void orc_qk_prep(float *x, uint32_t n_head, uint32_t head_dim, const uint16_t *w, uint32_t rotary_dim,
                 double theta, int llama3, uint32_t pos, float eps) {
    for (uint32_t h = 0; h < n_head; h++) {
        float *head = x + (uint64_t)h * head_dim;
        double ss = 0.0;
        for (uint32_t i = 0; i < head_dim; i++) ss += (double)head[i] * (double)head[i];
        const float scale = 1.0f / sqrtf((float)(ss / (double)head_dim) + eps);
        for (uint32_t i = 0; i < head_dim; i++) {
            uint32_t bits = (uint32_t)w[i] << 16;
            float wf;
            memcpy(&wf, &bits, 4);
            head[i] = head[i] * scale * (wf + 1.0f);
        }
        const uint32_t half = rotary_dim / 2u;
        for (uint32_t i = 0; i < half; i++) {
            const double inv = orc_inv_freq(i, rotary_dim, theta, llama3);
            const float c = cosf((float)((double)pos * inv));
            const float s = sinf((float)((double)pos * inv));
            const float a = head[i], b = head[i + half];
            head[i] = a * c - b * s;
            head[i + half] = b * c + a * s;
        }
    }
}

/* ---- Q8_0 matvec (the o_proj step after the attention) ----
 * sf37_q8_0_quantize_activation (sf37_ops.c:57-90): per 32-element block,
 * d = amax / 127 (the reference build's -ffast-math turns the division by
 * the constant into a product with its rounded reciprocal), iscale = 1 / d,
 * q = lrintf(iscale * x) clamped to [-128, 127]; an all-zero block has
 * d = 0 and q = 0.  sf37_q8_0_row_dot_prequant (sf37_ops.c:92-108): per
 * weight block (f16 scale + 32 int8, 34 bytes) an exact integer dot,
 * acc += isum * wscale * xscale in block order. */
void orc_q8_0_quantize(const float *x, int8_t *xq, float *xs, uint64_t n) {
    const uint64_t blocks = (n + 31u) / 32u;
    for (uint64_t b = 0; b < blocks; b++) {
        const uint64_t off = b * 32u;
        const uint64_t len = n - off < 32u ? n - off : 32u;
        float amax = 0.0f;
        for (uint64_t i = 0; i < len; i++) {
            const float a = fabsf(x[off + i]);
            if (a > amax) amax = a;
        }
        if (amax == 0.0f) {
            xs[b] = 0.0f;
            memset(xq + off, 0, 32);
            continue;
        }
        const float d = amax * (1.0f / 127.0f);
        const float is = 1.0f / d;
        xs[b] = d;
        for (uint64_t i = 0; i < len; i++) {
            int v = (int)lrintf(is * x[off + i]);
            if (v > 127) v = 127;
            if (v < -128) v = -128;
            xq[off + i] = (int8_t)v;
        }
        for (uint64_t i = len; i < 32u; i++) xq[off + i] = 0;
    }
}

void orc_q8_0_matvec(float *out, const uint8_t *w, uint64_t in_dim, uint64_t out_dim, const float *x) {
    const uint64_t blocks = (in_dim + 31u) / 32u;
    int8_t *xq = (int8_t *)malloc(blocks * 32u);
    float *xs = (float *)malloc(blocks * sizeof(float));
    if (!xq || !xs) abort();
    orc_q8_0_quantize(x, xq, xs, in_dim);
    for (uint64_t r = 0; r < out_dim; r++) {
        const uint8_t *row = w + r * blocks * 34u;
        float acc = 0.0f;
        for (uint64_t b = 0; b < blocks; b++) {
            const uint8_t *blk = row + b * 34u;
            const float ws = orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const int8_t *wq = (const int8_t *)(blk + 2);
            const uint64_t len = in_dim - b * 32u < 32u ? in_dim - b * 32u : 32u;
            int isum = 0;
            for (uint64_t i = 0; i < len; i++) isum += (int)wq[i] * (int)xq[b * 32u + i];
            acc += (float)isum * ws * xs[b];
        }
        out[r] = acc;
    }
    free(xs);
    free(xq);
}
