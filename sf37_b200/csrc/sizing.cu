// Decode cache sizing: the rules by which the reference engine sizes its
// per-layer KV caches (cuda_decode_state_init, sf37.c:3189-3216, with
// cuda_sliding_cache_cap 3067-3081, cuda_sliding_cache_prefill_cap
// 3083-3091, cuda_decode_kv_bytes_for_cap 3093-3096 and the free-memory
// tiers of cuda_prefill_default_chunk 5131-5140), and the pure form of the
// managed-memory policy (sf37_cuda.cu:1766-1800).  Host code only: these
// decide how much HBM the caches take and whether a sliding layer's ring is
// large enough for an exact chunked prefill.
#include <cstring>

#include "kv_internal.cuh"

using sf37kv::set_error;

namespace {

constexpr uint32_t kWindow = 512;           // SF37_SLIDING_WINDOW (sf37.c:60)
constexpr uint32_t kSlidingMax = 8192;      // SF37_CUDA_SLIDING_CACHE_MAX (sf37.c:72)
constexpr uint32_t kCtxMax = 262144;        // SF37_CTX (sf37.c:38)

uint32_t align_up(uint32_t v, uint32_t a) {
    const uint32_t rem = v % a;
    if (rem == 0) return v;
    if (v > UINT32_MAX - (a - rem)) return UINT32_MAX;
    return v + (a - rem);
}

uint32_t window_for(uint32_t ctx) {
    uint32_t w = kWindow;
    if (w > ctx) w = ctx;
    return w ? w : 1u;
}

}  // namespace

extern "C" uint32_t sf37kv_sliding_cache_cap(uint32_t ctx_size, uint32_t prefill_cap) {
    if (ctx_size == 0) return 1;
    const uint32_t w = window_for(ctx_size);
    uint64_t want = (uint64_t)w + prefill_cap;
    if (want > ctx_size) want = ctx_size;
    if (want == 0) want = 1;
    want = align_up((uint32_t)want, 256u);
    if (want > ctx_size) want = ctx_size;
    if (want > kSlidingMax) want = kSlidingMax;
    if (want < w) want = w;
    return (uint32_t)want;
}

extern "C" uint32_t sf37kv_sliding_prefill_cap(uint32_t ctx_size, uint32_t cache_cap) {
    if (cache_cap == 0) return 0;
    const uint32_t w = window_for(ctx_size);
    if (ctx_size <= w) return cache_cap;
    if (cache_cap <= w) return 1;
    return cache_cap - w;
}

extern "C" uint64_t sf37kv_kv_cache_bytes(uint32_t cap, uint32_t kv_heads, uint32_t head_dim, int dtype) {
    if (dtype != SF37KV_F16 && dtype != SF37KV_F32) return 0;
    return (uint64_t)cap * kv_heads * head_dim * 2u * (uint64_t)dtype;
}

extern "C" uint32_t sf37kv_prefill_default_chunk(uint64_t free_bytes) {
    const uint64_t gib = 1073741824ull;
    if (free_bytes >= 24ull * gib) return 4096;
    if (free_bytes >= 12ull * gib) return 2048;
    if (free_bytes >= 6ull * gib) return 1024;
    return 512;
}

extern "C" int sf37kv_plan_caches(uint32_t ctx_size, uint32_t prefill_chunk, uint32_t n_layers,
                                  uint32_t kv_heads, uint32_t head_dim, int dtype, sf37kv_cache_plan *plan) {
    if (!plan) return set_error(SF37KV_EINVAL, "plan_caches: plan is NULL");
    if (n_layers > SF37KV_PLAN_MAX_LAYERS)
        return set_error(SF37KV_EINVAL, "plan_caches: %u layers exceed %d", n_layers, SF37KV_PLAN_MAX_LAYERS);
    if (dtype != SF37KV_F16 && dtype != SF37KV_F32)
        return set_error(SF37KV_EINVAL, "plan_caches: unknown dtype %d", dtype);
    memset(plan, 0, sizeof(*plan));
    if (ctx_size == 0) ctx_size = 1;
    if (ctx_size > kCtxMax) ctx_size = kCtxMax;
    plan->ctx_size = ctx_size;
    plan->sliding_cap = sf37kv_sliding_cache_cap(ctx_size, prefill_chunk);
    plan->prefill_cap = sf37kv_sliding_prefill_cap(ctx_size, plan->sliding_cap);
    if (plan->prefill_cap == 0) plan->prefill_cap = 1;
    plan->window = window_for(ctx_size);
    for (uint32_t il = 0; il < n_layers; il++) {
        const bool full = (il % 4u) == 0u;  // layer_is_full (sf37.c:1983-1985)
        plan->cap[il] = full ? ctx_size : plan->sliding_cap;
        plan->sliding[il] = full ? 0u : 1u;
        if (full) plan->full_layers++;
        else plan->sliding_layers++;
        plan->kv_cache_bytes += sf37kv_kv_cache_bytes(plan->cap[il], kv_heads, head_dim, dtype);
    }
    return SF37KV_OK;
}

extern "C" int sf37kv_managed_kv_policy(uint64_t kv_cache_bytes, uint64_t context_bytes, uint64_t free_bytes,
                                        uint64_t total_bytes) {
    if (kv_cache_bytes == 0) return 0;
    const uint64_t gib = 1073741824ull;
    if (kv_cache_bytes >= 8ull * gib) return 1;
    if (context_bytes < 8ull * gib) return 0;
    uint64_t reserve = total_bytes / 4u;
    if (reserve < 8ull * gib) reserve = 8ull * gib;
    if (reserve > 40ull * gib) reserve = 40ull * gib;
    if (context_bytes > free_bytes) return 1;
    return free_bytes - context_bytes < reserve;
}
