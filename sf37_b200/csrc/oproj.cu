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
// while those copies are in flight, then each of its 8 warps walks its rows
// with a three-stage row pipeline (16 rows, 139 KB, in flight per SM): 8 dp4a per block, a float accumulator per lane
// and one warp reduction per row.  One launch covers many layers.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "kv_internal.cuh"
#include "../../include/sf37_cuda_kv.h"

namespace sf37kv {

extern unsigned long long g_launches;

namespace {


struct OprojJob {
    const uint8_t *w;
    const float *x;
    float *out;
    uint32_t cta_begin;  // first CTA of this job
    uint64_t red_off;    // float offset of this layer's partial in the peers' buffers
};

struct OprojParams {
    OprojJob job[kMaxJobs];
    uint32_t n_jobs;
    uint32_t in_dim, blocks, row_bytes, out_dim;
    uint32_t rows_per_cta, ctas_per_job;
    uint64_t row_stride;  // bytes between weight rows (>= row_bytes: a column slice)
    GatherDev red;        // world > 0: partial sums go to every rank (sf37kv_oproj_q8_0_shard)
};

constexpr uint32_t kMaxRowsPerCta = 1024;

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// kWarps warps per CTA, kStages rows in flight per warp (8 x 3 for rows up
// to 8.7 KB, fewer for wider rows so the stages fit in shared memory).
template <int kWarps, int kStages>
__global__ void __launch_bounds__(kWarps * 32) oproj_q8_0_kernel(const __grid_constant__ OprojParams P) {
    extern __shared__ __align__(16) uint8_t smem[];
    const uint32_t blocks = P.blocks, row_bytes = P.row_bytes;
    // x codes by block pair p (blocks 2p, 2p+1) at 80 p: the 16-byte pad
    // makes a lane's 16-byte reads of its pair bank-conflict free.
    int8_t *xq = reinterpret_cast<int8_t *>(smem);                        // [blocks/2][80]
    float *xs = reinterpret_cast<float *>(smem + blocks * 40u);           // [blocks]
    uint8_t *stage0 = smem + blocks * 44u;                                // [warps][stages][row_bytes]
    float *osm = reinterpret_cast<float *>(stage0 + (uint32_t)kWarps * kStages * row_bytes);  // [rows]

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
            const uint8_t *src = J.w + (uint64_t)row * P.row_stride;
            const uint32_t dst = stage_addr + (k % kStages) * row_bytes;
            for (uint32_t c = lane; c < chunks16; c += 32u) cp_async16(dst + c * 16u, src + c * 16u);
        }
        cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < kStages - 1; s++) issue(s);

    // Quantize x while the first rows load: sf37_q8_0_quantize_activation
    // (sf37_ops.c:57-90).  Eight lanes per 32-element block (a float4 each),
    // all of a thread's loads issued before any use.
    {
        constexpr int kPer = 8;  // blocks per 8-lane group per pass
        const uint32_t grp = threadIdx.x >> 3, sub = threadIdx.x & 7u, n_grp = kWarps * 4u;
        for (uint32_t b0 = grp; b0 < blocks; b0 += n_grp * kPer) {
            float4 v[kPer];
#pragma unroll
            for (int u = 0; u < kPer; u++) {
                const uint32_t b = b0 + (uint32_t)u * n_grp;
                v[u] = b < blocks ? reinterpret_cast<const float4 *>(J.x + b * 32u)[sub]
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kPer; u++) {
                const uint32_t b = b0 + (uint32_t)u * n_grp;
                float amax = fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
                if (b >= blocks) continue;
                uint32_t packed = 0;
                float d = 0.f;
                if (amax > 0.f) {
                    d = amax * (1.0f / 127.0f);
                    const float is = 1.0f / d;
                    const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        int q = __float2int_rn(is * e[c]);
                        q = q > 127 ? 127 : (q < -128 ? -128 : q);
                        packed |= ((uint32_t)q & 0xffu) << (8 * c);
                    }
                }
                *reinterpret_cast<uint32_t *>(xq + (b >> 1) * 80u + (b & 1u) * 32u + sub * 4u) = packed;
                if (sub == 0) xs[b] = d;
            }
        }
    }
    __syncthreads();

    for (uint32_t k = 0; k < n_mine; k++) {
        cp_async_wait<kStages - 2>();
        __syncwarp();
        issue(k + kStages - 1);
        const uint8_t *row = my_stage + (k % kStages) * row_bytes;
        // Lane handles block pairs p = lane, lane + 32, ...: 68 bytes starting
        // 4-byte aligned (17 words, stride 17 words across lanes: no bank
        // conflicts).  Block 2p: f16 scale in bytes 0-1, codes in bytes
        // 2-33 (funnel-shifted words); block 2p+1: scale in bytes 34-35,
        // codes in words 9-16.
        float acc = 0.f;
        const uint32_t *rw = reinterpret_cast<const uint32_t *>(row);
        for (uint32_t p = lane; p < blocks / 2u; p += 32u) {
            uint32_t w[17];
#pragma unroll
            for (int i = 0; i < 17; i++) w[i] = rw[p * 17u + i];
            const int4 *xp = reinterpret_cast<const int4 *>(xq + p * 80u);
            const int4 x0 = xp[0], x1 = xp[1], x2 = xp[2], x3 = xp[3];
            const float2 sx = *reinterpret_cast<const float2 *>(xs + 2u * p);
            int s0 = 0, s1 = 0;
            s0 = __dp4a((int)__funnelshift_r(w[0], w[1], 16), x0.x, s0);
            s0 = __dp4a((int)__funnelshift_r(w[1], w[2], 16), x0.y, s0);
            s0 = __dp4a((int)__funnelshift_r(w[2], w[3], 16), x0.z, s0);
            s0 = __dp4a((int)__funnelshift_r(w[3], w[4], 16), x0.w, s0);
            s0 = __dp4a((int)__funnelshift_r(w[4], w[5], 16), x1.x, s0);
            s0 = __dp4a((int)__funnelshift_r(w[5], w[6], 16), x1.y, s0);
            s0 = __dp4a((int)__funnelshift_r(w[6], w[7], 16), x1.z, s0);
            s0 = __dp4a((int)__funnelshift_r(w[7], w[8], 16), x1.w, s0);
            s1 = __dp4a((int)w[9], x2.x, s1);
            s1 = __dp4a((int)w[10], x2.y, s1);
            s1 = __dp4a((int)w[11], x2.z, s1);
            s1 = __dp4a((int)w[12], x2.w, s1);
            s1 = __dp4a((int)w[13], x3.x, s1);
            s1 = __dp4a((int)w[14], x3.y, s1);
            s1 = __dp4a((int)w[15], x3.z, s1);
            s1 = __dp4a((int)w[16], x3.w, s1);
            const float ws0 = __half2float(__ushort_as_half((unsigned short)(w[0] & 0xffffu)));
            const float ws1 = __half2float(__ushort_as_half((unsigned short)(w[8] >> 16)));
            acc += (float)s0 * ws0 * sx.x;
            acc += (float)s1 * ws1 * sx.y;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            if (P.red.world) osm[warp + k * kWarps] = acc;
            else J.out[r0 + warp + k * kWarps] = acc;
        }
    }
    cp_async_wait<0>();
    if (P.red.world) {
        // Row-parallel layers: this CTA's partial rows go to every rank's
        // buffer (coalesced NVLink stores); the last CTA of the launch raises
        // this rank's epoch flag everywhere (as the decode gather does).
        __syncthreads();
        const uint32_t nr = r1 - r0;
        for (uint32_t i = threadIdx.x; i < nr; i += blockDim.x) {
            const float v = osm[i];
            J.out[r0 + i] = v;
            for (uint32_t p = 0; p < P.red.world; p++)
                if (p != P.red.rank) P.red.peer[p][J.red_off + r0 + i] = v;
        }
        // publish: system acq_rel atomic per CTA, one fence before the flags
        __syncthreads();
        uint32_t prev = 0;
        if (threadIdx.x == 0)
            asm volatile("atom.acq_rel.sys.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(P.red.done) : "memory");
        if (threadIdx.x == 0 && prev == P.red.total_groups - 1u) {
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            for (uint32_t p = 0; p < P.red.world; p++) {
                uint32_t *f = P.red.peer_flags[p] + P.red.rank;
                asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(P.red.epoch) : "memory");
            }
            *P.red.done = 0u;
        }
    }
}

size_t oproj_smem(uint32_t blocks, uint32_t row_bytes, int warps, int stages) {
    return (size_t)blocks * 44u + (size_t)warps * stages * row_bytes + kMaxRowsPerCta * 4u;
}

struct OprojConfig {
    int warps, stages;
    void (*kernel)(OprojParams);
};
const OprojConfig kConfigs[] = {{8, 3, oproj_q8_0_kernel<8, 3>},
                                {8, 2, oproj_q8_0_kernel<8, 2>},
                                {4, 2, oproj_q8_0_kernel<4, 2>}};

}  // namespace

// One launch per 64 layers sharing in_dim / out_dim.  row_stride: bytes
// between weight rows; red / red_off: row-parallel partial sums to peers.
int oproj_q8_0(const sf37kv_oproj_layer *layers, uint32_t n, uint32_t in_dim, uint32_t out_dim,
               cudaStream_t stream, uint64_t row_stride = 0, const GatherDev *red = nullptr,
               const uint64_t *red_off = nullptr) {
    if (n == 0) return SF37KV_OK;
    if (!layers) return set_error(SF37KV_EINVAL, "oproj: layers is NULL");
    if (in_dim == 0 || in_dim % 256u || out_dim == 0)
        return set_error(SF37KV_EUNSUPPORTED, "oproj: in_dim %u must be a positive multiple of 256", in_dim);
    const uint32_t blocks = in_dim / 32u, row_bytes = blocks * 34u;
    if (row_stride == 0) row_stride = row_bytes;
    if (row_stride < row_bytes || row_stride % 16u)
        return set_error(SF37KV_EINVAL, "oproj: row stride %llu must be >= %u and a multiple of 16",
                         (unsigned long long)row_stride, row_bytes);
    if (red && n > (uint32_t)kMaxJobs)
        return set_error(SF37KV_EINVAL, "oproj: at most %d layers per row-parallel call", kMaxJobs);
    for (uint32_t i = 0; i < n; i++) {  // every argument check before any CUDA call
        const sf37kv_oproj_layer &L = layers[i];
        if (!L.weights || !L.x || !L.out)
            return set_error(SF37KV_EINVAL, "oproj: layer %u has a NULL pointer", i);
        if (((uintptr_t)L.weights | (uintptr_t)L.x) & 15u)
            return set_error(SF37KV_EINVAL, "oproj: layer %u weights and x must be 16-byte aligned", i);
    }
    const OprojConfig *cfg = nullptr;
    size_t smem = 0;
    for (const OprojConfig &c : kConfigs) {
        smem = oproj_smem(blocks, row_bytes, c.warps, c.stages);
        if (smem <= 227u * 1024u) {
            cfg = &c;
            break;
        }
    }
    if (!cfg)
        return set_error(SF37KV_EUNSUPPORTED, "oproj: in_dim %u needs %zu bytes of shared memory", in_dim, smem);
    static size_t attr[3] = {0, 0, 0};
    const int ci = (int)(cfg - kConfigs);
    if (smem > attr[ci]) {
        if (int rc = check_cuda(cudaFuncSetAttribute(cfg->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)smem),
                                "oproj smem attribute"))
            return rc;
        attr[ci] = smem;
    }
    // Rows per CTA: the split of each layer that fills whole waves best
    // (fewest waves per unit of work), as the decode planning does.
    // (occupancy cached per config and shared-memory size: the query costs
    // host time on every call otherwise)
    static size_t occ_smem[3] = {0, 0, 0};
    static int occ[3] = {0, 0, 0};
    if (occ_smem[ci] != smem) {
        int per = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, cfg->kernel, cfg->warps * 32, smem) != cudaSuccess ||
            per < 1) {
            (void)cudaGetLastError();
            per = 1;
        }
        occ[ci] = per;
        occ_smem[ci] = smem;
    }
    const int per_sm = occ[ci];
    for (uint32_t base = 0; base < n; base += kMaxJobs) {
        const uint32_t m = std::min<uint32_t>(n - base, kMaxJobs);
        const uint64_t slots = (uint64_t)num_sms() * per_sm;
        uint64_t best_c = (out_dim + kMaxRowsPerCta - 1) / kMaxRowsPerCta;
        double best = 1e30;
        const uint64_t max_c = std::max<uint64_t>(1, out_dim / cfg->warps);
        const uint64_t min_c = (out_dim + kMaxRowsPerCta - 1) / kMaxRowsPerCta;
        for (uint64_t c = min_c; c <= std::max(max_c, min_c) && c <= 4096; c++) {
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
        P.row_stride = row_stride;
        if (red) {
            P.red = *red;
            P.red.total_groups = m * P.ctas_per_job;
        }
        for (uint32_t i = 0; i < m; i++) {
            const sf37kv_oproj_layer &L = layers[base + i];
            P.job[i] = OprojJob{(const uint8_t *)L.weights, L.x, L.out, i * P.ctas_per_job,
                                red_off ? red_off[base + i] : 0};
        }
        const unsigned grid = m * P.ctas_per_job;
        cfg->kernel<<<grid, cfg->warps * 32, smem, stream>>>(P);
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

extern "C" int sf37kv_oproj_q8_0_shard(const sf37kv_oproj_layer *layers, uint32_t n_layers, uint32_t in_dim,
                                       uint32_t out_dim, uint64_t row_stride, const sf37kv_peer_gather *g,
                                       uint32_t epoch, void *stream) {
    GatherDev d;
    if (int rc = gather_dev(g, epoch, &d)) return rc;
    if (n_layers == 0 || n_layers > (uint32_t)kMaxJobs)
        return set_error(SF37KV_EINVAL, "oproj_shard: 1..%d layers per call", kMaxJobs);
    sf37kv_oproj_layer L[kMaxJobs];
    uint64_t off[kMaxJobs];
    const uint64_t n = (uint64_t)n_layers * out_dim;
    for (uint32_t i = 0; i < n_layers; i++) {
        off[i] = ((uint64_t)(epoch & 1u) * g->world + g->rank) * n + (uint64_t)i * out_dim;
        L[i] = layers[i];
        L[i].out = (float *)g->peer_buf[g->rank] + off[i];
    }
    return oproj_q8_0(L, n_layers, in_dim, out_dim, stream ? (cudaStream_t)stream : current_stream(), row_stride,
                      &d, off);
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
