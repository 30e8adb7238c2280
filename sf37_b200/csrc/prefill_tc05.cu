// tcgen05 (5th-generation tensor core) chunked prefill for f16 caches and
// bf16 queries.  Semantics: attention_prefill_heads128_warp_kernel
// (sf37_cuda.cu:3163-3239), as the mma.sync path in prefill_tc.cu.
//
// One CTA per (128 query rows, KV head).  The GQA group is folded into the
// M dimension: row r = hl * T + tl holds query head hl of the group for
// token tl of the block (T = 128 / G tokens), so every K/V tile feeds all G
// heads in one 128-row UMMA.  Per 128-key tile:
//   S[128 x 128]  = Q . K^T   8 x tcgen05.mma kind::f16 (M128 N128 K16),
//                             A = Q, B = K, both K-major in shared memory,
//                             accumulator in TMEM columns [0, 128);
//   softmax       thread r owns TMEM lane r (= row r): tcgen05.ld of its
//                 128 scores, mask, running max (log2 domain, raised only by
//                 > 8), exp2, row sum, P (f16) back to shared memory;
//   O[128 x 128] += P . V     8 x tcgen05.mma, A = P (K-major), B = V
//                             (MN-major: V rows are keys), accumulator in
//                             TMEM columns [128, 256).
// Shared-memory operands use the canonical 128-byte-swizzled layout: a tile
// is two 64-column halves, each [rows][128 B] with 16-byte chunk c of row r
// stored at chunk c ^ (r & 7); descriptor SBO = 1024 B (8-row groups), and
// for MN-major V the two d-halves are LBO = 16 KB apart.
//
// Every mbarrier wait is bounded (about 2 s of clock64 cycles): on timeout
// the CTA records an error in a device flag, stops issuing work, frees its
// TMEM and exits, so a fault in this kernel cannot hang the GPU.
#include <cmath>

#include "kv_internal.cuh"

namespace sf37kv {

extern unsigned long long g_launches;
int *device_error_flag();

struct Tc05Params {
    const __half *k, *v;
    const uint16_t *q;  // bf16 [n_tok][q_heads][128]
    const float *gate;  // [n_tok][q_heads] or nullptr
    float *out;         // [n_tok][q_heads][128]
    int *err;
    uint32_t pos0, n_tok, cap, sliding, window;
    uint32_t q_heads, kv_heads, group, tpt;  // tpt = 128 / group tokens per CTA
    float qscale;
};

namespace tc05 {

constexpr uint32_t kHalf = 16384;  // one 64-column half of a 128-row tile
constexpr uint32_t kTile = 2 * kHalf;
constexpr long long kWaitCycles = 4000000000ll;

__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: f32 accumulate, f16 A and B, A K-major,
// B K-major (b_mn = 0) or MN-major (b_mn = 1), N = 128, M = 128.
__host__ __device__ constexpr uint32_t idesc(uint32_t b_mn) {
    return (1u << 4) | (b_mn << 16) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar));
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;"); }

// Bounded parity wait; returns false on timeout.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t phase) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(bar), "r"(phase));
        if (ok) return true;
        if (clock64() - t0 > kWaitCycles) return false;
    }
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
        "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]),
        "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]),
        "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31]));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;"); }

__device__ __forceinline__ void cp16(uint32_t s, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(g));
}
// Byte offset of 16-byte chunk c (0..15) of row r in a swizzled 128-row tile.
__device__ __forceinline__ uint32_t tile_off(uint32_t r, uint32_t c) {
    return (c >> 3) * kHalf + r * 128u + (((c & 7u) ^ (r & 7u)) << 4);
}
__device__ __forceinline__ uint32_t start_of(uint32_t p, const Tc05Params &P) {
    const uint32_t have = p + 1u;
    uint32_t s = have > P.cap ? have - P.cap : 0u;
    if (P.sliding && have > P.window && have - P.window > s) s = have - P.window;
    return s;
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

}  // namespace tc05

__global__ void __launch_bounds__(128, 1) prefill_tc05_kernel(const __grid_constant__ Tc05Params P) {
    using namespace tc05;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    // 1024-byte aligned operand tiles: Q, K, V, P.
    const uint32_t s0 = ((uint32_t)__cvta_generic_to_shared(smem_raw) + 1023u) & ~1023u;
    const uint32_t sQ = s0, sK = s0 + kTile, sV = s0 + 2 * kTile, sP = s0 + 3 * kTile;
    const uint32_t bar_s = (uint32_t)__cvta_generic_to_shared(&bars[0]);
    const uint32_t bar_o = (uint32_t)__cvta_generic_to_shared(&bars[1]);
    const uint32_t tid = threadIdx.x, warp = tid >> 5;
    const uint32_t T = P.tpt;
    const uint32_t nblk = (P.n_tok + T - 1) / T;
    const uint32_t blk = nblk - 1u - blockIdx.x;  // longest causal ranges first
    const uint32_t kvh = blockIdx.y;
    const uint32_t tok0 = blk * T;
    const uint32_t tok_last = min(tok0 + T - 1u, P.n_tok - 1u);

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_s));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_o));
        asm volatile("fence.mbarrier_init.release.cluster;");
        abort_sh = 0;
    }
    if (warp == 0) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_base_sh);
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(dst));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // Q tile: row r = hl * T + tl, bf16 -> f16, swizzled.
    const uint32_t r = tid;
    const uint32_t hl = r / T, tl = r - hl * T;
    const uint32_t tok = tok0 + tl;
    const uint32_t qh = kvh * P.group + hl;
    {
        const uint32_t tq = min(tok, P.n_tok - 1u);
        const uint4 *src = reinterpret_cast<const uint4 *>(P.q + ((uint64_t)tq * P.q_heads + qh) * 128u);
        uint8_t *gsm = smem_raw + (sQ - (uint32_t)__cvta_generic_to_shared(smem_raw));
#pragma unroll
        for (uint32_t c = 0; c < 16; c++) {
            const uint4 x = __ldg(src + c);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
            uint4 h;
            uint32_t *ho = &h.x;
#pragma unroll
            for (int i = 0; i < 4; i++)
                ho[i] = pack_h2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
            *reinterpret_cast<uint4 *>(gsm + tile_off(r, c)) = h;
        }
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t t_s = tmem, t_o = tmem + 128u;
    const uint32_t lane_off = (warp * 32u) << 16;

    const uint32_t p_row = P.pos0 + tok;
    const uint32_t s_row = start_of(p_row, P);
    const uint32_t kbeg = start_of(P.pos0 + tok0, P);
    const uint32_t kend = P.pos0 + tok_last + 1u;
    const uint32_t ntiles = (kend - kbeg + 127u) / 128u;
    const uint64_t row_bytes = (uint64_t)P.kv_heads * 256u;
    const char *kg = reinterpret_cast<const char *>(P.k) + kvh * 256u;
    const char *vg = reinterpret_cast<const char *>(P.v) + kvh * 256u;
    uint8_t *gsm_p = smem_raw + (sP - (uint32_t)__cvta_generic_to_shared(smem_raw));

    float m = -INFINITY, l = 0.f;
    uint32_t phase = 0;
    bool ok = true;
    for (uint32_t j = 0; j < ntiles && ok; j++) {
        const uint32_t k0 = kbeg + j * 128u;
        // K and V tiles: 128 keys x 16 chunks each; 16 + 16 per thread per pass.
        for (uint32_t c = tid; c < 2048u; c += 128u) {
            const uint32_t kr = c >> 4, ch = c & 15u;
            uint32_t kp = k0 + kr;
            if (kp >= kend) kp = kbeg;
            const uint64_t go = (uint64_t)(kp % P.cap) * row_bytes + ch * 16u;
            cp16(sK + tile_off(kr, ch), kg + go);
            cp16(sV + tile_off(kr, ch), vg + go);
        }
        asm volatile("cp.async.commit_group;");
        asm volatile("cp.async.wait_group 0;");
        fence_async_smem();
        fence_before();
        __syncthreads();
        fence_after();
        if (tid == 0) {
#pragma unroll
            for (uint32_t kk = 0; kk < 8; kk++) {
                const uint32_t off = (kk >> 2) * kHalf + (kk & 3u) * 32u;
                mma(t_s, sdesc(sQ + off, 16, 1024), sdesc(sK + off, 16, 1024), idesc(0), kk > 0);
            }
            commit(bar_s);
        }
        if (!wait_bar(bar_s, phase)) {
            atomicExch(&abort_sh, 1);
        }
        fence_after();
        if (__syncthreads_or(abort_sh)) {
            ok = false;
            break;
        }
        // Scores of this thread's row.
        float s[128];
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) {
            float v[32];
            tmem_ld32(t_s + lane_off + q4 * 32u, v);
#pragma unroll
            for (int i = 0; i < 32; i++) s[q4 * 32 + i] = v[i];
        }
        tmem_wait_ld();
        float mx = -INFINITY;
        const bool full = k0 >= start_of(P.pos0 + tok_last, P) && k0 + 127u <= P.pos0 + tok0;
#pragma unroll
        for (int i = 0; i < 128; i++) {
            float x = s[i] * P.qscale;
            if (!full) {
                const uint32_t kp = k0 + (uint32_t)i;
                if (kp < s_row || kp > p_row || kp >= kend) x = -INFINITY;
            }
            s[i] = x;
            mx = fmaxf(mx, x);
        }
        const bool need = mx > m + 8.0f;
        if (__any_sync(0xffffffffu, need)) {
            const float mn = need ? mx : m;
            const float alpha = (m == -INFINITY || mn == -INFINITY) ? 0.f : fast_exp2(m - mn);
            if (j > 0) {  // O holds earlier tiles: rescale this warp's rows in TMEM
#pragma unroll
                for (int q4 = 0; q4 < 4; q4++) {
                    float v[32];
                    tmem_ld32(t_o + lane_off + q4 * 32u, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] *= need ? alpha : 1.0f;
                    tmem_st32(t_o + lane_off + q4 * 32u, v);
                }
                tmem_wait_st();
            }
            if (need) {
                l *= alpha;
                m = mn;
            }
        }
        const float mu = m == -INFINITY ? 0.f : m;
#pragma unroll
        for (uint32_t c = 0; c < 16; c++) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float p0 = fast_exp2(s[c * 8 + 2 * i] - mu), p1 = fast_exp2(s[c * 8 + 2 * i + 1] - mu);
                l += p0 + p1;
                w[i] = pack_h2(p0, p1);
            }
            *reinterpret_cast<uint4 *>(gsm_p + tile_off(r, c)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_async_smem();
        fence_before();
        __syncthreads();
        fence_after();
        if (tid == 0) {
#pragma unroll
            for (uint32_t kk = 0; kk < 8; kk++) {
                const uint32_t offp = (kk >> 2) * kHalf + (kk & 3u) * 32u;
                mma(t_o, sdesc(sP + offp, 16, 1024), sdesc(sV + kk * 2048u, kHalf, 1024), idesc(1),
                    (j > 0 || kk > 0) ? 1u : 0u);
            }
            commit(bar_o);
        }
        if (!wait_bar(bar_o, phase)) atomicExch(&abort_sh, 1);
        fence_after();
        phase ^= 1u;
        if (__syncthreads_or(abort_sh)) {
            ok = false;
            break;
        }
    }

    if (ok) {
        // tcgen05.ld is warp-collective: every lane loads, only real rows store.
        const bool store = tok < P.n_tok;
        const float gt = (store && P.gate) ? sigmoid_dev(P.gate[(uint64_t)tok * P.q_heads + qh]) : 1.f;
        const float f = l > 0.f ? gt / l : 0.f;
        float4 *op = reinterpret_cast<float4 *>(P.out + ((uint64_t)min(tok, P.n_tok - 1u) * P.q_heads + qh) * 128u);
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) {
            float v[32];
            if (ntiles > 0) {
                tmem_ld32(t_o + lane_off + q4 * 32u, v);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.f;
            }
            if (store)
#pragma unroll
                for (int i = 0; i < 8; i++)
                    op[q4 * 8 + i] = make_float4(v[4 * i] * f, v[4 * i + 1] * f, v[4 * i + 2] * f, v[4 * i + 3] * f);
        }
    }
    if (!ok && tid == 0) atomicExch(P.err, 1);
    fence_before();
    __syncthreads();
    fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
}

int prefill_tc05(const sf37kv_cache *cache, const void *q, const float *gate, float *out, uint32_t pos0,
                 uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads, cudaStream_t stream, bool *handled) {
    *handled = false;
    if (kv_heads == 0 || q_heads % kv_heads) return SF37KV_OK;
    const uint32_t G = q_heads / kv_heads;
    if (G == 0 || G > 128 || 128 % G) return SF37KV_OK;
    if (((uintptr_t)cache->k_cache | (uintptr_t)cache->v_cache | (uintptr_t)q) & 15u) return SF37KV_OK;
    int *err = device_error_flag();
    if (!err) return SF37KV_OK;
    Tc05Params P{(const __half *)cache->k_cache, (const __half *)cache->v_cache, (const uint16_t *)q, gate,
                 out, err, pos0, n_tok, cache->cap, cache->sliding, cache->window, q_heads, kv_heads, G,
                 128u / G, 1.4426950408889634f / sqrtf(128.0f)};
    const size_t sm = 4 * tc05::kTile + 1024;
    cudaFuncSetAttribute(prefill_tc05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    dim3 grid((n_tok + P.tpt - 1) / P.tpt, kv_heads);
    prefill_tc05_kernel<<<grid, 128, sm, stream>>>(P);
    g_launches++;
    if (int rc = check_cuda(cudaGetLastError(), "prefill tcgen05 launch")) return rc;
    *handled = true;
    return SF37KV_OK;
}

}  // namespace sf37kv
