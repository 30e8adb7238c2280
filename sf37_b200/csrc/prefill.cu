// Chunked-prefill attention: token t of a chunk is a causal query at
// pos0 + t over rows start_at(pos0+t) .. pos0+t (attention_prefill_heads128
// _warp_kernel, sf37_cuda.cu:3163-3239; entry point 3241-3317).
//
// This file holds the entry points, the dispatch and the query-per-job
// fallback (every token runs the split-K decode kernels; K/V are re-read from
// L2 per token), used only for shapes the tile kernels do not take (head_dim
// other than 128, other groups).  The tile kernels: prefill_tc05.cu (tcgen05,
// f16 caches + bf16 q), prefill_tc.cu (mma.sync: f16 caches with wrapping
// rings or f32 q, and fp32 caches + fp32 q, the engine's drop-in call).
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "kv_internal.cuh"
#include "../../include/sf37_cuda_kv.h"

namespace sf37kv {

extern unsigned long long g_launches;

int prefill_tc05(const sf37kv_cache *cache, const void *q, const float *gate, float *out, uint32_t pos0,
                 uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads, cudaStream_t stream, bool *handled);
int prefill_tc(const sf37kv_cache *cache, const void *q, int q_type, const float *gate, float *out,
               uint32_t pos0, uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads,
               cudaStream_t stream, bool *handled);
int prefill_tc32(const sf37kv_cache *cache, const float *q, const float *gate, float *out, uint32_t pos0,
                 uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads, cudaStream_t stream, bool *handled);

// f32 caches: the tensor-core kernel where its shape conditions hold, else
// every token as a split-K decode job.
static int prefill_f32_any(const sf37kv_cache *c, const float *q, const float *gate, float *out, uint32_t pos0,
                           uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                           cudaStream_t stream);

__global__ static void bf16_to_f32_kernel(const uint16_t *src, float *dst, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = __uint_as_float((uint32_t)src[i] << 16);
}

static float *g_qconv = nullptr;
static uint64_t g_qconv_elems = 0;

// Query-per-job prefill (f32 queries).
static int prefill_jobs(const sf37kv_cache *c, const float *q, const float *gate, float *out,
                        uint32_t pos0, uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads,
                        uint32_t head_dim, int dtype, cudaStream_t stream) {
    const uint64_t q_dim = (uint64_t)q_heads * head_dim;
    AttnJob jobs[kMaxJobs];
    for (uint32_t base = 0; base < n_tok; base += kMaxJobs) {
        uint32_t m = 0;
        for (uint32_t t = base; t < n_tok && m < (uint32_t)kMaxJobs; t++, m++) {
            const uint32_t pos = pos0 + t;
            jobs[m] = AttnJob{c->k_cache, c->v_cache, q + (uint64_t)t * q_dim,
                              gate ? gate + (uint64_t)t * q_heads : nullptr, out + (uint64_t)t * q_dim,
                              start_at(pos, c->cap, c->sliding, c->window), pos + 1u, c->cap};
        }
        if (int rc = attention_jobs(jobs, m, q_heads, kv_heads, head_dim, dtype, stream)) return rc;
    }
    return SF37KV_OK;
}

}  // namespace sf37kv

using namespace sf37kv;

extern "C" int sf37kv_prefill(const sf37kv_cache *cache, const void *q, int q_type, const float *gate,
                              float *out, uint32_t pos0, uint32_t n_tok, uint32_t q_heads,
                              uint32_t kv_heads, uint32_t head_dim, int dtype, void *stream) {
    if (!cache || !q || !out || cache->cap == 0)
        return set_error(SF37KV_EINVAL, "prefill: null argument or cap 0");
    if (q_type != SF37KV_Q_F32 && q_type != SF37KV_Q_BF16)
        return set_error(SF37KV_EINVAL, "prefill: unknown q type %d", q_type);
    if (n_tok == 0) return SF37KV_OK;
    if (cache->sliding) {
        // The chunk's own append must not have overwritten a row that its
        // first token attends to: the oldest row still in the ring,
        // pos0 + n_tok - cap, may not be newer than that token's window
        // start (the reference engine keeps chunks within cap - window,
        // sf37.c:3083-3091, 3197-3200).
        const uint64_t end = (uint64_t)pos0 + n_tok;
        const uint64_t oldest = end > cache->cap ? end - cache->cap : 0;
        const uint64_t first = (cache->window && pos0 + 1u > cache->window) ? pos0 + 1u - cache->window : 0;
        if (oldest > first)
            return set_error(SF37KV_EINVAL,
                             "prefill: sliding ring of %u rows cannot hold a %u-token chunk with its %u-row window "
                             "(needs cap >= window + n_tok - 1)",
                             cache->cap, n_tok, cache->window);
    }
    cudaStream_t s = stream ? (cudaStream_t)stream : current_stream();
    if (dtype == SF37KV_F16 && head_dim == 128) {
        bool handled = false;
        if (q_type == SF37KV_Q_BF16)
            if (int rc = prefill_tc05(cache, q, gate, out, pos0, n_tok, q_heads, kv_heads, s, &handled))
                return rc;
        if (!handled)
        if (int rc = prefill_tc(cache, q, q_type, gate, out, pos0, n_tok, q_heads, kv_heads, s, &handled))
            return rc;
        if (handled) return SF37KV_OK;
    }
    const float *qf = (const float *)q;
    if (q_type == SF37KV_Q_BF16) {
        const uint64_t n = (uint64_t)n_tok * q_heads * head_dim;
        if (n > g_qconv_elems) {
            if (g_qconv) {
                cudaDeviceSynchronize();
                cudaFree(g_qconv);
                g_qconv = nullptr;
                g_qconv_elems = 0;
            }
            if (int rc = check_cuda(cudaMalloc(&g_qconv, n * 4), "prefill q buffer")) return rc;
            g_qconv_elems = n;
        }
        bf16_to_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const uint16_t *)q, g_qconv, n);
        g_launches++;
        if (int rc = check_cuda(cudaGetLastError(), "bf16 convert launch")) return rc;
        qf = g_qconv;
    }
    if (dtype == SF37KV_F32) return prefill_f32_any(cache, qf, gate, out, pos0, n_tok, q_heads, kv_heads, head_dim, s);
    return prefill_jobs(cache, qf, gate, out, pos0, n_tok, q_heads, kv_heads, head_dim, dtype, s);
}

namespace sf37kv {
static int prefill_f32_any(const sf37kv_cache *c, const float *q, const float *gate, float *out, uint32_t pos0,
                           uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                           cudaStream_t stream) {
    if (head_dim == 128) {
        bool handled = false;
        if (int rc = prefill_tc32(c, q, gate, out, pos0, n_tok, q_heads, kv_heads, stream, &handled)) return rc;
        if (handled) return SF37KV_OK;
    }
    return prefill_jobs(c, q, gate, out, pos0, n_tok, q_heads, kv_heads, head_dim, SF37KV_F32, stream);
}
}  // namespace sf37kv

extern "C" int sf37_cuda_attention_prefill_heads(sf37_cuda_tensor *out_heads, const sf37_cuda_tensor *q,
                                                 const sf37_cuda_tensor *k_cache,
                                                 const sf37_cuda_tensor *v_cache,
                                                 const sf37_cuda_tensor *head_gate, uint32_t pos0,
                                                 uint32_t n_tok, uint32_t cache_cap, uint32_t q_heads,
                                                 uint32_t kv_heads, uint32_t head_dim, int sliding,
                                                 uint32_t window) {
    // Validation as sf37_cuda.cu:3254-3267.
    if (!out_heads || !q || !k_cache || !v_cache || !head_gate || n_tok == 0 || cache_cap == 0 ||
        kv_heads == 0 || q_heads % kv_heads != 0 || head_dim == 0)
        return 0;
    const uint64_t q_dim = (uint64_t)q_heads * head_dim, kv_dim = (uint64_t)kv_heads * head_dim;
    if (n_tok > UINT64_MAX / q_dim / 4 || out_heads->bytes < (uint64_t)n_tok * q_dim * 4 ||
        q->bytes < (uint64_t)n_tok * q_dim * 4 || head_gate->bytes < (uint64_t)n_tok * q_heads * 4 ||
        k_cache->bytes < (uint64_t)cache_cap * kv_dim * 4 || v_cache->bytes < (uint64_t)cache_cap * kv_dim * 4)
        return 0;
    sf37kv_cache c{k_cache->ptr, v_cache->ptr, cache_cap, (uint32_t)(sliding != 0), window, 0};
    if (prefill_f32_any(&c, (const float *)q->ptr, (const float *)head_gate->ptr, (float *)out_heads->ptr,
                        pos0, n_tok, q_heads, kv_heads, head_dim, current_stream())) {
        fprintf(stderr, "sf37: attention_prefill_heads failed: %s\n", sf37kv_last_error());
        return 0;
    }
    return 1;
}

extern "C" int sf37_cuda_store_kv_cache_batch(sf37_cuda_tensor *k_cache, sf37_cuda_tensor *v_cache,
                                              const sf37_cuda_tensor *k, const sf37_cuda_tensor *v,
                                              uint32_t pos0, uint32_t n_tok, uint32_t cache_cap,
                                              uint32_t kv_dim) {
    // Validation as sf37_cuda.cu:6382-6390.
    if (!k_cache || !v_cache || !k || !v || n_tok == 0 || cache_cap == 0 || kv_dim == 0) return 0;
    if (n_tok > UINT64_MAX / kv_dim / 4 || k->bytes < (uint64_t)n_tok * kv_dim * 4 ||
        v->bytes < (uint64_t)n_tok * kv_dim * 4 || k_cache->bytes < (uint64_t)cache_cap * kv_dim * 4 ||
        v_cache->bytes < (uint64_t)cache_cap * kv_dim * 4)
        return 0;
    AppendJob j{k_cache->ptr, v_cache->ptr, (const float *)k->ptr, (const float *)v->ptr, pos0, n_tok,
                cache_cap};
    if (append_jobs(&j, 1, kv_dim, SF37KV_F32, current_stream())) {
        fprintf(stderr, "sf37: store_kv_cache_batch failed: %s\n", sf37kv_last_error());
        return 0;
    }
    return 1;
}
