// Q8_0 matvec of the attention output projection -- the step right after the
// decode attention (o_proj, sf37.c:3367-3369 via sf37_cuda_matvec_q8_0_mapped,
// sf37_cuda.cu:3319-3349 + 3433-3461; CPU form sf37_ops.c:57-123).
//
// Weights: per output row, in_dim/32 blocks of 34 bytes (f16 scale, then 32
// int8).  The activation x (the gated attention heads, f32) is quantized to
// the same 32-element blocks (scale d = amax/127, q = rint(x/d)), and
// out[r] = sum_b (float)dot(wq_b, xq_b) * wscale_b * xscale_b.
//
// B200 layout: the weights are the only HBM stream (35.7 MB per layer at
// 4096 x 8192), so the kernel is HBM-bound.  A CTA owns a contiguous run of
// rows of one layer.  It first queues cp.async copies of its warps' first
// rows into shared memory, then quantizes x (from L2) into shared memory
// while those copies are in flight, then each warp walks its rows with a
// two-stage row pipeline: 8 dp4a per block, a float accumulator per lane
// and one warp reduction per row.  One launch covers many layers.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "kv_internal.cuh"
#include "../../include/sf37_cuda_kv.h"

namespace sf37kv {

extern unsigned long long g_launches;

namespace {

constexpr int kWarps = 4;
constexpr int kStages = 2;

struct OprojJob {
    const uint8_t *w;
    const float *x;
    float *out;
    uint32_t cta_begin;  // first CTA of this job
};

struct OprojParams {
    OprojJob job[kMaxJobs];
    uint32_t n_jobs;
    uint32_t in_dim, blocks, row_bytes, out_dim;
    uint32_t rows_per_cta, ctas_per_job;
};

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kWarps * 32) oproj_q8_0_kernel(const __grid_constant__ OprojParams P) {
    extern __shared__ __align__(16) uint8_t smem[];
    const uint32_t blocks = P.blocks, row_bytes = P.row_bytes;
    int8_t *xq = reinterpret_cast<int8_t *>(smem);                        // [blocks][32]
    float *xs = reinterpret_cast<float *>(smem + blocks * 32u);           // [blocks]
    uint8_t *stage0 = smem + blocks * 36u;                                // [warps][stages][row_bytes]

    const uint32_t j = blockIdx.x / P.ctas_per_job;
    const OprojJob &J = P.job[j];
    const uint32_t chunk = blockIdx.x - j * P.ctas_per_job;
    const uint32_t r0 = chunk * P.rows_per_cta;
    const uint32_t r1 = min(r0 + P.rows_per_cta, P.out_dim);
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint8_t *my_stage = stage0 + (uint32_t)warp * kStages * row_bytes;
    const uint32_t stage_addr = (uint32_t)__cvta_generic_to_shared(my_stage);
    const uint32_t chunks16 = row_bytes / 16u;

    // rows of this warp: r0 + warp, r0 + warp + kWarps, ...
    const uint32_t n_mine = r0 + warp < r1 ? (r1 - r0 - warp + kWarps - 1) / kWarps : 0u;
    auto issue = [&](uint32_t k) {
        if (k < n_mine) {
            const uint32_t row = r0 + warp + k * kWarps;
            const uint8_t *src = J.w + (uint64_t)row * row_bytes;
            const uint32_t dst = stage_addr + (k % kStages) * row_bytes;
            for (uint32_t c = lane; c < chunks16; c += 32u) cp_async16(dst + c * 16u, src + c * 16u);
        }
        cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < kStages - 1; s++) issue(s);

    // Quantize x while the first rows load: sf37_q8_0_quantize_activation
    // (sf37_ops.c:57-90), one warp per 32-element block.
    for (uint32_t b = warp; b < blocks; b += kWarps) {
        const float v = J.x[b * 32u + lane];
        float amax = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        int q = 0;
        float d = 0.f;
        if (amax > 0.f) {
            d = amax * (1.0f / 127.0f);
            const float is = 1.0f / d;
            q = __float2int_rn(is * v);
            q = q > 127 ? 127 : (q < -128 ? -128 : q);
        }
        xq[b * 32u + lane] = (int8_t)q;
        if (lane == 0) xs[b] = d;
    }
    __syncthreads();

    for (uint32_t k = 0; k < n_mine; k++) {
        cp_async_wait<kStages - 2>();
        __syncwarp();
        issue(k + kStages - 1);
        const uint8_t *row = my_stage + (k % kStages) * row_bytes;
        float acc = 0.f;
        for (uint32_t b = lane; b < blocks; b += 32u) {
            const uint8_t *blk = row + b * 34u;
            const float ws = __half2float(*reinterpret_cast<const __half *>(blk));
            // 32 int8 weights at blk + 2: 4-byte aligned when b is odd,
            // else shifted by 2 bytes (funnel-shift adjacent words).
            int32_t wv[8];
            if (b & 1u) {
                const int32_t *p = reinterpret_cast<const int32_t *>(blk + 2);
#pragma unroll
                for (int i = 0; i < 8; i++) wv[i] = p[i];
            } else {
                const uint32_t *p = reinterpret_cast<const uint32_t *>(blk);
                uint32_t prev = p[0];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const uint32_t nxt = p[i + 1];
                    wv[i] = (int32_t)__funnelshift_r(prev, nxt, 16);
                    prev = nxt;
                }
            }
            const int4 xa = *reinterpret_cast<const int4 *>(xq + b * 32u);
            const int4 xb = *reinterpret_cast<const int4 *>(xq + b * 32u + 16u);
            int isum = 0;
            isum = __dp4a(wv[0], xa.x, isum);
            isum = __dp4a(wv[1], xa.y, isum);
            isum = __dp4a(wv[2], xa.z, isum);
            isum = __dp4a(wv[3], xa.w, isum);
            isum = __dp4a(wv[4], xb.x, isum);
            isum = __dp4a(wv[5], xb.y, isum);
            isum = __dp4a(wv[6], xb.z, isum);
            isum = __dp4a(wv[7], xb.w, isum);
            acc += (float)isum * ws * xs[b];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) J.out[r0 + warp + k * kWarps] = acc;
    }
    cp_async_wait<0>();
}

size_t oproj_smem(uint32_t blocks, uint32_t row_bytes) {
    return (size_t)blocks * 36u + (size_t)kWarps * kStages * row_bytes;
}

}  // namespace

// One launch for n layers sharing in_dim / out_dim.
int oproj_q8_0(const sf37kv_oproj_layer *layers, uint32_t n, uint32_t in_dim, uint32_t out_dim,
               cudaStream_t stream) {
    if (n == 0) return SF37KV_OK;
    if (!layers) return set_error(SF37KV_EINVAL, "oproj: layers is NULL");
    if (in_dim == 0 || in_dim % 256u || out_dim == 0)
        return set_error(SF37KV_EUNSUPPORTED, "oproj: in_dim %u must be a positive multiple of 256", in_dim);
    const uint32_t blocks = in_dim / 32u, row_bytes = blocks * 34u;
    const size_t smem = oproj_smem(blocks, row_bytes);
    if (smem > 227u * 1024u)
        return set_error(SF37KV_EUNSUPPORTED, "oproj: in_dim %u needs %zu bytes of shared memory", in_dim, smem);
    static size_t attr = 0;
    if (smem > attr) {
        if (int rc = check_cuda(cudaFuncSetAttribute(oproj_q8_0_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)smem),
                                "oproj smem attribute"))
            return rc;
        attr = smem;
    }
    // Rows per CTA: the split of each layer that fills whole waves best
    // (fewest waves per unit of work), as the decode planning does.
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, oproj_q8_0_kernel, kWarps * 32, smem) != cudaSuccess ||
        per_sm < 1) {
        (void)cudaGetLastError();
        per_sm = 1;
    }
    for (uint32_t base = 0; base < n; base += kMaxJobs) {
        const uint32_t m = std::min<uint32_t>(n - base, kMaxJobs);
        const uint64_t slots = (uint64_t)num_sms() * per_sm;
        uint64_t best_c = 1;
        double best = 1e30;
        const uint64_t max_c = std::max<uint64_t>(1, out_dim / kWarps);
        for (uint64_t c = 1; c <= max_c && c <= 4096; c++) {
            const double cost = (double)((c * m + slots - 1) / slots) / (double)c;
            if (cost < best * 0.95) {
                best = cost;
                best_c = c;
            }
        }
        OprojParams P;
        memset(&P, 0, sizeof(P));
        P.n_jobs = m;
        P.in_dim = in_dim;
        P.blocks = blocks;
        P.row_bytes = row_bytes;
        P.out_dim = out_dim;
        P.rows_per_cta = (uint32_t)((out_dim + best_c - 1) / best_c);
        P.ctas_per_job = (out_dim + P.rows_per_cta - 1) / P.rows_per_cta;
        for (uint32_t i = 0; i < m; i++) {
            const sf37kv_oproj_layer &L = layers[base + i];
            if (!L.weights || !L.x || !L.out)
                return set_error(SF37KV_EINVAL, "oproj: layer %u has a NULL pointer", base + i);
            if (((uintptr_t)L.weights | (uintptr_t)L.x) & 15u)
                return set_error(SF37KV_EINVAL, "oproj: layer %u weights and x must be 16-byte aligned", base + i);
            P.job[i] = OprojJob{(const uint8_t *)L.weights, L.x, L.out, i * P.ctas_per_job};
        }
        const unsigned grid = m * P.ctas_per_job;
        oproj_q8_0_kernel<<<grid, kWarps * 32, smem, stream>>>(P);
        g_launches++;
        if (int rc = check_cuda(cudaGetLastError(), "oproj launch")) return rc;
    }
    return SF37KV_OK;
}

// Activation quantization alone (the reference's quantize_q8_0_f32_kernel,
// sf37_cuda.cu:3319-3349; CPU sf37_ops.c:57-90): exposed so the int8 codes
// can be checked bit for bit.
__global__ void q8_0_quantize_kernel(const float *x, int8_t *xq, float *xs, uint32_t blocks) {
    const uint32_t b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31u;
    if (b >= blocks) return;
    const float v = x[b * 32u + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int q = 0;
    float d = 0.f;
    if (amax > 0.f) {
        d = amax * (1.0f / 127.0f);
        const float is = 1.0f / d;
        q = __float2int_rn(is * v);
        q = q > 127 ? 127 : (q < -128 ? -128 : q);
    }
    xq[b * 32u + lane] = (int8_t)q;
    if (lane == 0) xs[b] = d;
}

}  // namespace sf37kv

using namespace sf37kv;

extern "C" int sf37kv_oproj_q8_0(const sf37kv_oproj_layer *layers, uint32_t n_layers, uint32_t in_dim,
                                 uint32_t out_dim, void *stream) {
    return oproj_q8_0(layers, n_layers, in_dim, out_dim, stream ? (cudaStream_t)stream : current_stream());
}

extern "C" int sf37kv_q8_0_quantize(const float *x, int8_t *xq, float *xscale, uint64_t n, void *stream) {
    if (!x || !xq || !xscale) return set_error(SF37KV_EINVAL, "q8_0 quantize: NULL pointer");
    if (n == 0 || n % 32u) return set_error(SF37KV_EUNSUPPORTED, "q8_0 quantize: n must be a multiple of 32");
    const uint32_t blocks = (uint32_t)(n / 32u);
    cudaStream_t s = stream ? (cudaStream_t)stream : current_stream();
    q8_0_quantize_kernel<<<(blocks + 7u) / 8u, 256, 0, s>>>(x, xq, xscale, blocks);
    g_launches++;
    return check_cuda(cudaGetLastError(), "q8_0 quantize launch");
}

// Drop-in for sf37_cuda_matvec_q8_0 (sf37_cuda.h:134-137, sf37_cuda.cu:3708-3734):
// tensor handles, byte-size validation, 1 = success.
extern "C" int sf37_cuda_matvec_q8_0(sf37_cuda_tensor *out, const sf37_cuda_tensor *weights, uint64_t in_dim,
                                     uint64_t out_dim, const sf37_cuda_tensor *x) {
    if (!out || !weights || !x) return 0;
    const uint64_t blocks = (in_dim + 31u) / 32u;
    if (out->bytes < out_dim * sizeof(float) || x->bytes < in_dim * sizeof(float) ||
        weights->bytes < out_dim * blocks * 34u)
        return 0;
    if (in_dim > 0xffffffffull || out_dim > 0xffffffffull) return 0;
    sf37kv_oproj_layer L{weights->ptr, (const float *)x->ptr, (float *)out->ptr};
    if (int rc = oproj_q8_0(&L, 1, (uint32_t)in_dim, (uint32_t)out_dim, current_stream())) {
        (void)rc;
        fprintf(stderr, "sf37: q8_0 matvec failed: %s\n", sf37kv_last_error());
        return 0;
    }
    return 1;
}
