// K/V append: token t of a batch lands in ring slot (pos0 + t) % cap
// (store_kv_cache_batch_kernel, sf37_cuda.cu:6355-6401).
//
// One CTA per (job, token) row; each thread moves 4 consecutive elements of
// K and of V with 128-bit loads, so one decode append (kv_dim 1024) is one
// CTA of 256 threads and a batch of layers is one launch.  For f16 caches
// the f32 row is rounded to nearest even (__float2half2_rn), 64-bit stores.
// HBM-bound: 2*kv_dim*(4 + elem) bytes per row.
#include "kv_internal.cuh"

namespace sf37kv {

extern unsigned long long g_launches;

struct AppendParams {
    AppendJob job[kMaxJobs];
    uint32_t row_begin[kMaxJobs + 1];  // prefix sum of n_tok
    uint32_t n_jobs;
    uint32_t kv_dim;
};

template <typename T>
__device__ __forceinline__ void store4(T *dst, float4 x);

template <>
__device__ __forceinline__ void store4<float>(float *dst, float4 x) {
    *reinterpret_cast<float4 *>(dst) = x;
}

template <>
__device__ __forceinline__ void store4<__half>(__half *dst, float4 x) {
    __half2 a = __floats2half2_rn(x.x, x.y);
    __half2 b = __floats2half2_rn(x.z, x.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(dst) = u;
}

__device__ __forceinline__ void store1(float *dst, float x) { *dst = x; }
__device__ __forceinline__ void store1(__half *dst, float x) { *dst = __float2half_rn(x); }

template <typename T, bool kVec>
__global__ void __launch_bounds__(256) append_kernel(const __grid_constant__ AppendParams P) {
    const uint32_t row = blockIdx.x;
    uint32_t j = 0;
    while (j + 1 < P.n_jobs && P.row_begin[j + 1] <= row) j++;
    const AppendJob &J = P.job[j];
    const uint32_t t = row - P.row_begin[j];
    // With n_tok > cap several tokens share a slot; the last one wins, as in
    // a sequential append (kv_cache_push order).  Earlier ones write nothing.
    if ((uint64_t)t + J.cap < J.n_tok) return;
    const uint64_t slot = (uint64_t)((J.pos0 + t) % J.cap);
    const uint32_t kv_dim = P.kv_dim;
    T *kc = reinterpret_cast<T *>(J.k_cache) + slot * kv_dim;
    T *vc = reinterpret_cast<T *>(J.v_cache) + slot * kv_dim;
    const float *k = J.k + (uint64_t)t * kv_dim;
    const float *v = J.v + (uint64_t)t * kv_dim;
    if (kVec) {
        for (uint32_t i = threadIdx.x * 4u; i < kv_dim; i += blockDim.x * 4u) {
            store4<T>(kc + i, __ldg(reinterpret_cast<const float4 *>(k + i)));
            store4<T>(vc + i, __ldg(reinterpret_cast<const float4 *>(v + i)));
        }
    } else {
        for (uint32_t i = threadIdx.x; i < kv_dim; i += blockDim.x) {
            store1(kc + i, k[i]);
            store1(vc + i, v[i]);
        }
    }
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

int append_jobs(const AppendJob *jobs, uint32_t n, uint32_t kv_dim, int dtype,
                cudaStream_t stream) {
    if (dtype != SF37KV_F32 && dtype != SF37KV_F16)
        return set_error(SF37KV_EINVAL, "append: unknown cache dtype %d", dtype);
    if (kv_dim == 0) return set_error(SF37KV_EINVAL, "append: kv_dim is 0");
    for (uint32_t base = 0; base < n; base += kMaxJobs) {
        AppendParams P;
        P.n_jobs = 0;
        P.kv_dim = kv_dim;
        uint32_t rows = 0;
        bool vec = (kv_dim % 4u) == 0;
        for (uint32_t i = base; i < n && i < base + kMaxJobs; i++) {
            const AppendJob &J = jobs[i];
            if (!J.k_cache || !J.v_cache || !J.k || !J.v || J.cap == 0)
                return set_error(SF37KV_EINVAL, "append: job %u has a null pointer or cap 0", i);
            if (J.n_tok == 0) continue;
            if ((uint64_t)rows + J.n_tok > 0x7fffffffull)
                return set_error(SF37KV_EINVAL, "append: too many rows in one call");
            vec = vec && aligned16(J.k) && aligned16(J.v) &&
                  ((uintptr_t)J.k_cache % (dtype == SF37KV_F32 ? 16u : 8u)) == 0 &&
                  ((uintptr_t)J.v_cache % (dtype == SF37KV_F32 ? 16u : 8u)) == 0;
            P.job[P.n_jobs] = J;
            P.row_begin[P.n_jobs] = rows;
            P.n_jobs++;
            rows += J.n_tok;
        }
        if (P.n_jobs == 0) continue;
        P.row_begin[P.n_jobs] = rows;
        const unsigned threads = vec ? (kv_dim / 4u < 256u ? ((kv_dim / 4u + 31u) & ~31u) : 256u)
                                     : 256u;
        if (dtype == SF37KV_F32) {
            if (vec) append_kernel<float, true><<<rows, threads, 0, stream>>>(P);
            else append_kernel<float, false><<<rows, threads, 0, stream>>>(P);
        } else {
            if (vec) append_kernel<__half, true><<<rows, threads, 0, stream>>>(P);
            else append_kernel<__half, false><<<rows, threads, 0, stream>>>(P);
        }
        g_launches++;
        if (int rc = check_cuda(cudaGetLastError(), "append launch")) return rc;
    }
    return SF37KV_OK;
}

}  // namespace sf37kv

using namespace sf37kv;

extern "C" int sf37kv_append(const sf37kv_append_layer *layers, uint32_t n_layers,
                             uint32_t kv_dim, int dtype, void *stream) {
    if (!layers && n_layers) return set_error(SF37KV_EINVAL, "append: layers is NULL");
    AppendJob jobs[kMaxJobs];
    cudaStream_t s = stream ? (cudaStream_t)stream : current_stream();
    for (uint32_t base = 0; base < n_layers; base += kMaxJobs) {
        uint32_t m = 0;
        for (uint32_t i = base; i < n_layers && m < (uint32_t)kMaxJobs; i++, m++) {
            const sf37kv_append_layer &L = layers[i];
            jobs[m] = AppendJob{L.cache.k_cache, L.cache.v_cache, L.k, L.v, L.pos0, L.n_tok,
                                L.cache.cap};
        }
        if (int rc = append_jobs(jobs, m, kv_dim, dtype, s)) return rc;
    }
    return SF37KV_OK;
}
