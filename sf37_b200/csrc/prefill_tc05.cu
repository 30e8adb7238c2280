// tcgen05 (5th-generation tensor core) chunked prefill for f16 caches and
// bf16 queries.  Semantics: attention_prefill_heads128_warp_kernel
// (sf37_cuda.cu:3163-3239), as the mma.sync path in prefill_tc.cu.
//
// One CTA per (two Q tiles, KV head).  The GQA group is folded into M: Q
// tile row r = hl * T + tl holds query head hl of the group for token tl of
// the tile (T = 128 / G tokens), so one 128-row UMMA serves all G heads of a
// KV head.  The two Q tiles (A, B: consecutive token blocks) share every K/V
// tile and ping-pong so one tile's softmax overlaps the other's MMAs.
//
// Warp roles (576 threads):
//   warps 0-7  softmax of tile A, warps 8-15 softmax of tile B.  Two threads
//              share each row: warp q (+4) owns TMEM lane quadrant q (rows
//              32q..32q+31) and score columns 0-63 (64-127).  Per key tile:
//              tcgen05.ld of the 64 scores, row max exchanged with the
//              partner warp through shared memory (pair barrier), lazy O
//              rescale in TMEM when the running max rises by more than 8
//              (log2 domain), exp2 (half on the MUFU unit, half by an FMA
//              polynomial), row sums, P (f16) written back into the first
//              64 TMEM columns of S with tcgen05.st;
//   warp 16    one elected thread issues tcgen05.mma kind::f16 (M128 N128
//              K16): S_t = Q_t K^T (A, B K-major in smem) and O_t += P_t V
//              (A = P from TMEM, V MN-major in smem); accumulators S_A, S_B,
//              O_A, O_B fill the 512 TMEM columns; tcgen05.commit -> mbarrier;
//   warp 17    one thread issues TMA tile loads (cp.async.bulk.tensor.2d,
//              single-CTA destination) of K and V tiles, each double-buffered, into
//              128B-swizzled shared memory as soon as the MMAs release them.
// Shared-memory operand tiles are two 64-column halves [rows][128 B] with
// 16-byte chunk c of row r at c ^ (r & 7) (the TMA 128B swizzle); UMMA
// descriptor SBO = 1024 B, and for MN-major V the d-halves are LBO = 16 KB
// apart.  Keys are read through the tensor maps at slot = position, so this
// kernel is used when the chunk does not wrap the ring (pos0 + n_tok <=
// cap); wrapping rings use the mma.sync kernel.
//
// Every mbarrier wait is bounded (about 2 s of clock64 cycles): on timeout
// the CTA records an error in a device flag, every role leaves its loop,
// TMEM is freed and the CTA exits, so a fault here cannot hang the GPU.
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "kv_internal.cuh"

namespace sf37kv {

extern unsigned long long g_launches;
int *device_error_flag();

struct Tc05Params {
    CUtensorMap kmap, vmap;  // [cap][kv_heads*128] f16, box 64 x 128 rows, 128B swizzle
    const uint16_t *q;  // bf16 [n_tok][q_heads][128]
    const float *gate;  // [n_tok][q_heads] or nullptr
    float *out;         // [n_tok][q_heads][128]
    int *err;
    uint32_t pos0, n_tok, cap, sliding, window;
    uint32_t q_heads, kv_heads, group, tpt;  // tpt = 128 / group tokens per Q tile
    float qscale;
};

namespace tc05 {

constexpr uint32_t kHalf = 16384;  // one 64-column half of a 128-row tile
constexpr uint32_t kTile = 2 * kHalf;
constexpr long long kWaitCycles = 4000000000ll;
// try_wait may suspend the thread up to this long (ns); it resumes as soon as
// the phase completes, so waiting warps do not steal issue slots.
constexpr uint32_t kSuspendNs = 100000;

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
// A operand from tensor memory (M x K, lane = row, two f16 per column).
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]));
}
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]));
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
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(bar), "r"(phase), "r"(kSuspendNs));
        if (ok) return true;
        if (clock64() - t0 > kWaitCycles) return false;
    }
}

// Warp-uniform wait: lane 0 polls, the result is broadcast, and the warp is
// converged afterwards (tcgen05.ld/st are .sync.aligned warp instructions).
__device__ __forceinline__ bool wait_bar_warp(uint32_t bar, uint32_t phase) {
    uint32_t ok = 1;
    if ((threadIdx.x & 31u) == 0) ok = wait_bar(bar, phase) ? 1u : 0u;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
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
// 2^x on the FMA pipe (to offload the MUFU unit, which half the softmax
// exponentials still use): x = i + f with i = rint(x) from the 1.5 * 2^23
// rounding trick, f in [-0.5, 0.5]; 2^f by a cubic fitted here (least
// squares on Chebyshev nodes, max relative error 7.5e-5, below the f16
// rounding P gets next); 2^i added to the exponent field.  x < -127 is
// clamped (the result then rounds to 0 in f16 anyway).
__device__ __forceinline__ float exp2_fma(float x) {
    x = fmaxf(x, -127.0f);
    const float t = x + 12582912.0f;
    const float f = x - (t - 12582912.0f);
    const float p = fmaf(fmaf(fmaf(0.05517162f, f, 0.24261113f), f, 0.69326097f), f, 0.99992806f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}



__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar));
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes));
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

}  // namespace tc05

// POLY: one in POLY exp2 evaluations of a row uses the FMA polynomial
// (exp2_fma), the others the MUFU unit (0 = MUFU only); balances the MUFU
// and issue limits of the softmax warps.
template <int POLY>
__global__ void __launch_bounds__(576, 1) prefill_tc05_kernel(const __grid_constant__ Tc05Params P) {
    using namespace tc05;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    enum { B_KFULL = 0, B_KEMPTY = 2, B_VFULL = 4, B_VEMPTY = 6, B_SFULL = 8, B_PFULL = 10, B_ODONE = 12,
           N_BARS = 14 };
    enum { T_QA = 0, T_K = 2, T_V = 4 };
    __shared__ __align__(8) uint64_t bars[N_BARS];
    __shared__ uint32_t tmem_base_sh;
    __shared__ volatile int abort_sh;
    __shared__ float xch[2][2][2][128];  // [parity][tile][half][row]: row max / sum exchange

    const uint32_t sraw = (uint32_t)__cvta_generic_to_shared(smem_raw);
    const uint32_t s0 = (sraw + 1023u) & ~1023u;
    uint8_t *gsm = smem_raw + (s0 - sraw);
    // tiles (32 KB each): Q_A, Q_B, K0, K1, V0, V1.  P_t lives in TMEM, in
    // the first 64 columns of S_t (two f16 per column).
    auto tile = [&](int i) { return s0 + (uint32_t)i * kTile; };
    auto bar = [&](int i) { return (uint32_t)__cvta_generic_to_shared(&bars[i]); };
    const uint32_t tid = threadIdx.x, warp = tid >> 5;
    const uint32_t T = P.tpt;
    const uint32_t nblk = (P.n_tok + 2u * T - 1u) / (2u * T);
    const uint32_t blk = nblk - 1u - blockIdx.x;  // longest causal ranges first
    const uint32_t kvh = blockIdx.y;
    const uint32_t tok0 = blk * 2u * T;           // first token of tile A
    const uint32_t tok_last = min(tok0 + 2u * T - 1u, P.n_tok - 1u);
    const uint32_t kbeg = start_of(P.pos0 + tok0, P);
    const uint32_t kend = P.pos0 + tok_last + 1u;
    const uint32_t ntiles = (kend - kbeg + 127u) / 128u;

    if (tid == 0) {
        for (int t = 0; t < 2; t++) {
            bar_init(bar(B_KFULL + t), 1);
            bar_init(bar(B_KEMPTY + t), 1);
            bar_init(bar(B_VFULL + t), 1);
            bar_init(bar(B_VEMPTY + t), 1);
            bar_init(bar(B_SFULL + t), 1);
            bar_init(bar(B_PFULL + t), 256);
            bar_init(bar(B_ODONE + t), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;");
        abort_sh = 0;
    }
    if (warp == 0) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_base_sh);
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(dst));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // Softmax warps 0-15: tile t_id = warp / 8; within a tile, warp q (+4 h)
    // owns TMEM lane quadrant q (rows 32q..32q+31) and column half h.  Each
    // row is shared by two threads (h = 0, 1), 64 score columns each.
    const uint32_t t_id = warp >> 3;
    const uint32_t hh = (warp >> 2) & 1u;
    const uint32_t r = ((warp & 3u) << 5) | (tid & 31u);
    const uint32_t hl = r / T, tl = r - hl * T;
    const uint32_t tok = tok0 + t_id * T + tl;
    const uint32_t qh = kvh * P.group + hl;
    if (warp < 16) {
        const uint32_t tq = min(tok, P.n_tok - 1u);
        const uint4 *src = reinterpret_cast<const uint4 *>(P.q + ((uint64_t)tq * P.q_heads + qh) * 128u);
        uint8_t *qt = gsm + (tile(T_QA + t_id) - s0);
#pragma unroll
        for (uint32_t c = 8u * hh; c < 8u * hh + 8u; c++) {
            const uint4 x = __ldg(src + c);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
            uint4 hv;
            uint32_t *ho = &hv.x;
#pragma unroll
            for (int i = 0; i < 4; i++)
                ho[i] = pack_h2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
            *reinterpret_cast<uint4 *>(qt + tile_off(r, c)) = hv;
        }
        fence_async_smem();
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = tmem_base_sh;

    if (warp == 17) {
        // ---------------- TMA loader: K and V double-buffered (buffer j % 2) ----------------
        if ((tid & 31u) == 0) {
            const int32_t x0 = (int32_t)(kvh * 128u);
            auto load = [&](int which, uint32_t j) {  // which: 0 = K, 1 = V
                const uint32_t b = j & 1u;
                const int32_t y = (int32_t)(kbeg + j * 128u);
                const uint32_t full = bar((which ? B_VFULL : B_KFULL) + b);
                const uint32_t dst = tile((which ? T_V : T_K) + b);
                const CUtensorMap *map = which ? &P.vmap : &P.kmap;
                bar_expect_tx(full, kTile);
                tma_load_2d(dst, map, x0, y, full);
                tma_load_2d(dst + kHalf, map, x0 + 64, y, full);
            };
            for (uint32_t j = 0; j < 2 && j < ntiles; j++) {
                load(0, j);
                load(1, j);
            }
            for (uint32_t j = 0; j + 2 < ntiles && !abort_sh; j++) {
                if (!wait_bar(bar(B_KEMPTY + (j & 1u)), (j >> 1) & 1u)) { abort_sh = 1; break; }
                load(0, j + 2);
                if (!wait_bar(bar(B_VEMPTY + (j & 1u)), (j >> 1) & 1u)) { abort_sh = 1; break; }
                load(1, j + 2);
            }
        }
    } else if (warp == 16) {
        // ---------------- MMA issuer ----------------
        // S_t(j+1)
        // overwrites the TMEM columns PV_t(j) reads P_t from; tcgen05.mma
        // operations issued by one thread execute in issue order.
        if ((tid & 31u) == 0) {
            auto issue_s = [&](uint32_t t, uint32_t j) {
                const uint32_t kt = tile(T_K + (j & 1u));
                fence_after();
#pragma unroll
                for (uint32_t kk = 0; kk < 8; kk++) {
                    const uint32_t off = (kk >> 2) * kHalf + (kk & 3u) * 32u;
                    mma(tmem + t * 128u, sdesc(tile(T_QA + t) + off, 16, 1024), sdesc(kt + off, 16, 1024),
                        idesc(0), kk > 0);
                }
                commit(bar(B_SFULL + t));
            };
            auto issue_pv = [&](uint32_t t, uint32_t j) {
                const uint32_t vt = tile(T_V + (j & 1u));
                fence_after();
#pragma unroll
                for (uint32_t kk = 0; kk < 8; kk++)
                    mma_ts(tmem + 256u + t * 128u, tmem + t * 128u + kk * 8u, sdesc(vt + kk * 2048u, kHalf, 1024),
                           idesc(1), (j > 0 || kk > 0) ? 1u : 0u);
                commit(bar(B_ODONE + t));
            };
            // Tile B starts one softmax later than tile A, so the two tiles'
            // softmaxes alternate and each overlaps the other tile's MMAs:
            // S_A0 | S_B0 PV_A0 S_A1 | PV_B0 S_B1 | PV_A1 S_A2 | PV_B1 S_B2 | ...
            bool bad = !wait_bar(bar(B_KFULL), 0);
            if (!bad) issue_s(0, 0);
            for (uint32_t j = 0; j < ntiles && !bad && !abort_sh; j++) {
                const bool more = j + 1 < ntiles;
                const uint32_t vb = j & 1u, vph = (j >> 1) & 1u;
                if (!wait_bar(bar(B_PFULL), j & 1u)) { bad = true; break; }
                if (j == 0) {
                    issue_s(1, 0);
                    commit(bar(B_KEMPTY));
                }
                if (!wait_bar(bar(B_VFULL + vb), vph)) { bad = true; break; }
                issue_pv(0, j);
                if (more) {
                    if (!wait_bar(bar(B_KFULL + ((j + 1) & 1u)), ((j + 1) >> 1) & 1u)) { bad = true; break; }
                    issue_s(0, j + 1);
                }
                if (!wait_bar(bar(B_PFULL + 1), j & 1u)) { bad = true; break; }
                issue_pv(1, j);
                commit(bar(B_VEMPTY + vb));
                if (more) {
                    issue_s(1, j + 1);
                    commit(bar(B_KEMPTY + ((j + 1) & 1u)));
                }
            }
            if (bad) abort_sh = 1;
        }
    } else {
        // ---------------- softmax (tile t_id, column half hh) ----------------
        const uint32_t lane_off = ((warp & 3u) * 32u) << 16;
        const uint32_t cb = 64u * hh;  // this thread's score / output columns
        const uint32_t t_s = tmem + t_id * 128u + lane_off, t_o = tmem + 256u + t_id * 128u + lane_off;
        const uint32_t pair_bar = 1u + t_id * 4u + (warp & 3u);  // the two warps sharing these rows
        // Pair barrier that also ORs a failure flag, so both warps of a pair
        // always take the same exit (a lone exit would strand the partner).
        auto pair_any = [&](bool v) -> bool {
            uint32_t rr;
            asm volatile(
                "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
                "bar.red.or.pred q, %2, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}\n"
                : "=r"(rr)
                : "r"((uint32_t)v), "r"(pair_bar));
            return rr != 0;
        };
        const uint32_t p_row = P.pos0 + tok;
        const uint32_t s_row = start_of(p_row, P);
        const uint32_t tt0 = tok0 + t_id * T, ttl = min(tt0 + T - 1u, P.n_tok - 1u);
        const uint32_t full_lo = start_of(P.pos0 + ttl, P), full_hi = P.pos0 + tt0;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        const float qs = P.qscale;
        // One pass over this thread's 64 scores of tile k0 with reference max
        // mu: P (packed f16) into w, sums into la, and the largest exponent
        // x = s * qs - mu (log2 units) into xm.
        auto pass = [&](uint32_t k0, bool full, float mu, uint32_t (&w)[2][16], float &la, float &xm) {
            float lb = 0.f, xa = -INFINITY, xb = -INFINITY;
            la = 0.f;
#pragma unroll
            for (int q2 = 0; q2 < 2; q2++) {
                float v[32];
                tmem_ld32(t_s + cb + q2 * 32u, v);
                tmem_wait_ld();
                if (full) {
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const float x0 = fmaf(v[2 * i], qs, -mu), x1 = fmaf(v[2 * i + 1], qs, -mu);
                        xa = fmaxf(xa, x0);
                        xb = fmaxf(xb, x1);
                        const float p0 = fast_exp2(x0);
                        const float p1 = (POLY > 0 && (i % (POLY > 0 ? POLY : 1)) == 0) ? exp2_fma(x1) : fast_exp2(x1);
                        la += p0;
                        lb += p1;
                        w[q2][i] = pack_h2(p0, p1);
                    }
                } else {
                    const uint32_t kb = k0 + cb + (uint32_t)(q2 * 32);
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const uint32_t kp = kb + 2u * i;
                        const bool ok0 = kp >= s_row && kp <= p_row && kp < kend;
                        const bool ok1 = kp + 1u >= s_row && kp + 1u <= p_row && kp + 1u < kend;
                        const float x0 = ok0 ? fmaf(v[2 * i], qs, -mu) : -INFINITY;
                        const float x1 = ok1 ? fmaf(v[2 * i + 1], qs, -mu) : -INFINITY;
                        xa = fmaxf(xa, x0);
                        xb = fmaxf(xb, x1);
                        const float p0 = fast_exp2(x0);
                        const float p1 = (POLY > 0 && (i % (POLY > 0 ? POLY : 1)) == 0) ? exp2_fma(x1) : fast_exp2(x1);
                        la += p0;
                        lb += p1;
                        w[q2][i] = pack_h2(p0, p1);
                    }
                }
            }
            la += lb;
            xm = fmaxf(xa, xb);
        };
        for (uint32_t j = 0; j < ntiles; j++) {
            const uint32_t k0 = kbeg + j * 128u;
            __syncwarp();
            const bool got_s = !abort_sh && wait_bar_warp(bar(B_SFULL + t_id), j & 1u);
            fence_after();
            // s_full(j) follows every earlier MMA of the issuing thread, so
            // PV_t(j-1) is complete: O_t is stable and P_t may be rewritten.
            const bool full = k0 >= full_lo && k0 + 127u <= full_hi;
            uint32_t w[2][16];
            float la = 0.f, xm = -INFINITY;
            const float mu0 = m == -INFINITY ? 0.f : m;
            if (got_s) pass(k0, full, mu0, w, la, xm);
            if (pair_any(!got_s)) { abort_sh = 1; ok = false; break; }
            // The running max only moves when some exponent exceeds 8 (or on
            // the first tile); then the row max is exchanged with the partner
            // half, O and l are rescaled and P is recomputed.
            const bool need = m == -INFINITY || xm > 8.0f;
            if (pair_any(need)) {
                xch[j & 1u][t_id][hh][r] = xm + mu0;
                pair_any(false);
                const float mx = fmaxf(xch[j & 1u][t_id][0][r], xch[j & 1u][t_id][1][r]);
                const bool row_need = mx > -INFINITY && (m == -INFINITY || mx > m + 8.0f);
                if (__any_sync(0xffffffffu, row_need)) {
                    const float alpha = (m == -INFINITY || !row_need) ? (row_need ? 0.f : 1.f) : fast_exp2(m - mx);
                    if (j > 0) {
#pragma unroll
                        for (int q2 = 0; q2 < 2; q2++) {
                            float v[32];
                            tmem_ld32(t_o + cb + q2 * 32u, v);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 32; i++) v[i] *= alpha;
                            tmem_st32(t_o + cb + q2 * 32u, v);
                        }
                        tmem_wait_st();
                    }
                    if (row_need) {
                        l *= alpha;
                        m = mx;
                    }
                    pass(k0, full, m == -INFINITY ? 0.f : m, w, la, xm);
                }
                pair_any(false);  // both halves have re-read S before P overwrites it
            }
            l += la;
            // keys cb .. cb+63 -> P columns cb/2 .. cb/2 + 31
            tmem_st16u(t_s + cb / 2u, w[0]);
            tmem_st16u(t_s + cb / 2u + 16u, w[1]);
            tmem_wait_st();
            fence_before();
            bar_arrive(bar(B_PFULL + t_id));  // P_t ready (S_t fully consumed)
        }
        const bool got_e = ok && !abort_sh && wait_bar_warp(bar(B_ODONE + t_id), (ntiles - 1) & 1u);
        if (ok) {
            xch[0][t_id][hh][r] = l;
            if (pair_any(!got_e)) ok = false;
        }
        if (ok) {
            fence_after();
            const float lt = xch[0][t_id][0][r] + xch[0][t_id][1][r];
            const bool store = tok < P.n_tok;
            const float gt = (store && P.gate) ? sigmoid_dev(P.gate[(uint64_t)tok * P.q_heads + qh]) : 1.f;
            const float f = lt > 0.f ? gt / lt : 0.f;
            float4 *op = reinterpret_cast<float4 *>(P.out + ((uint64_t)min(tok, P.n_tok - 1u) * P.q_heads + qh) * 128u + cb);
#pragma unroll
            for (int q2 = 0; q2 < 2; q2++) {
                float v[32];
                tmem_ld32(t_o + cb + q2 * 32u, v);
                tmem_wait_ld();
                if (store)
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        op[q2 * 8 + i] = make_float4(v[4 * i] * f, v[4 * i + 1] * f, v[4 * i + 2] * f, v[4 * i + 3] * f);
            }
        } else {
            abort_sh = 1;
        }
    }
    fence_before();
    __syncthreads();
    if (abort_sh && tid == 0) atomicExch(P.err, 1);
    fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
        else
            (void)cudaGetLastError();
    }
    return fn;
}

static bool make_map(CUtensorMap *map, const void *base, uint32_t kv_dim, uint32_t cap) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {kv_dim, cap};
    cuuint64_t strides[1] = {(cuuint64_t)kv_dim * 2u};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int prefill_tc05(const sf37kv_cache *cache, const void *q, const float *gate, float *out, uint32_t pos0,
                 uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads, cudaStream_t stream, bool *handled) {
    *handled = false;
    if (kv_heads == 0 || q_heads % kv_heads) return SF37KV_OK;
    const uint32_t G = q_heads / kv_heads;
    if (G == 0 || G > 128 || 128 % G) return SF37KV_OK;
    if ((uint64_t)pos0 + n_tok > cache->cap) return SF37KV_OK;  // ring wraps: mma.sync kernel
    if (((uintptr_t)cache->k_cache | (uintptr_t)cache->v_cache | (uintptr_t)q) & 15u) return SF37KV_OK;
    int *err = device_error_flag();
    if (!err) return SF37KV_OK;
    Tc05Params P;
    const uint32_t kv_dim = kv_heads * 128u;
    if (!make_map(&P.kmap, cache->k_cache, kv_dim, cache->cap) ||
        !make_map(&P.vmap, cache->v_cache, kv_dim, cache->cap))
        return SF37KV_OK;
    P.q = (const uint16_t *)q;
    P.gate = gate;
    P.out = out;
    P.err = err;
    P.pos0 = pos0;
    P.n_tok = n_tok;
    P.cap = cache->cap;
    P.sliding = cache->sliding;
    P.window = cache->window;
    P.q_heads = q_heads;
    P.kv_heads = kv_heads;
    P.group = G;
    P.tpt = 128u / G;
    P.qscale = 1.4426950408889634f / sqrtf(128.0f);
    const size_t sm = 6 * tc05::kTile + 1024;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(prefill_tc05_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        attr = true;
    }
    dim3 grid((n_tok + 2 * P.tpt - 1) / (2 * P.tpt), kv_heads);
    prefill_tc05_kernel<0><<<grid, 576, sm, stream>>>(P);
    g_launches++;
    if (int rc = check_cuda(cudaGetLastError(), "prefill tcgen05 launch")) return rc;
    *handled = true;
    return SF37KV_OK;
}

}  // namespace sf37kv
