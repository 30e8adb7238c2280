// Tensor-core chunked prefill for f16 caches and bf16 queries.
//
// Semantics as attention_prefill_heads128_warp_kernel (sf37_cuda.cu:3163-
// 3239): token t of the chunk is a causal query at p = pos0 + t over logical
// rows start_at(p) .. p (ring slot r % cap), out = softmax(q.K/sqrt(d)).V *
// sigmoid(gate[t][h]).
//
// Tiling (FlashAttention-2 style, GQA folded into the CTA): one CTA per
// (16-token block, KV head) with one warp per query head of the group, so
// all G heads share every K/V tile in shared memory.  Key tiles of 64 rows
// (K and V, 16 KB each) stream through a 3-stage cp.async ring; each warp
// computes S = Q K^T (16 x 64) and O += P V (16 x 128) with mma.sync
// m16n8k16 (f16 in, f32 accumulate), fragments loaded with ldmatrix (V
// transposed) from a chunk ^ (row & 7) swizzled layout (conflict free).
// The online softmax runs in the log2 domain on the accumulators and P is
// re-packed to f16 A fragments in registers.  bf16 queries are converted to
// f16 (exact for |q| in [2^-14, 65504]).
#include <cmath>

#include <cuda_bf16.h>

#include "kv_internal.cuh"

namespace sf37kv {

extern unsigned long long g_launches;

struct PrefillParams {
    const __half *k, *v;
    const uint16_t *q;  // bf16 [n_tok][q_heads][128]
    const float *gate;  // [n_tok][q_heads] or nullptr
    float *out;         // [n_tok][q_heads][128]
    uint32_t pos0, n_tok, cap, sliding, window;
    uint32_t q_heads, kv_heads;
    float qscale;       // log2(e)/sqrt(128)
};

namespace {

constexpr int kKeys = 64;             // keys per tile
constexpr int kStages = 3;
constexpr uint32_t kTileBytes = kKeys * 256;  // one of K or V

__device__ __forceinline__ void cp16(uint32_t s, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(g));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                    uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ uint32_t bf16x2_to_h2(uint32_t x) {
    const float lo = __uint_as_float(x << 16), hi = __uint_as_float(x & 0xffff0000u);
    return pack_h2(lo, hi);
}
__device__ __forceinline__ uint32_t start_of(uint32_t p, const PrefillParams &P) {
    const uint32_t have = p + 1u;
    uint32_t s = have > P.cap ? have - P.cap : 0u;
    if (P.sliding && have > P.window && have - P.window > s) s = have - P.window;
    return s;
}

}  // namespace

template <int NW>
__global__ void __launch_bounds__(NW * 32, 1) prefill_mma_kernel(const __grid_constant__ PrefillParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t nblk = (P.n_tok + 15u) >> 4;
    const uint32_t tb = nblk - 1u - blockIdx.x;  // longest causal ranges first
    const uint32_t kvh = blockIdx.y;
    const uint32_t h = kvh * NW + warp;           // query head of this warp
    const uint32_t tok0 = tb * 16u;
    const uint32_t tok_last = min(tok0 + 15u, P.n_tok - 1u);

    // Q fragments (rows = tokens tok0+g, tok0+g+8; 8 k-steps of 16 dims).
    uint32_t qa[8][4];
    {
        const uint32_t r0 = min(tok0 + g, P.n_tok - 1u), r1 = min(tok0 + g + 8u, P.n_tok - 1u);
        const uint32_t *q0 = reinterpret_cast<const uint32_t *>(P.q + ((uint64_t)r0 * P.q_heads + h) * 128u);
        const uint32_t *q1 = reinterpret_cast<const uint32_t *>(P.q + ((uint64_t)r1 * P.q_heads + h) * 128u);
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            qa[kk][0] = bf16x2_to_h2(q0[kk * 8 + t]);
            qa[kk][1] = bf16x2_to_h2(q1[kk * 8 + t]);
            qa[kk][2] = bf16x2_to_h2(q0[kk * 8 + 4 + t]);
            qa[kk][3] = bf16x2_to_h2(q1[kk * 8 + 4 + t]);
        }
    }
    const uint32_t prow[2] = {P.pos0 + tok0 + g, P.pos0 + tok0 + g + 8u};
    const uint32_t srow[2] = {start_of(prow[0], P), start_of(prow[1], P)};

    const uint32_t kbeg = start_of(P.pos0 + tok0, P);
    const uint32_t kend = P.pos0 + tok_last + 1u;
    const uint32_t ntiles = (kend - kbeg + kKeys - 1) / kKeys;
    // Tiles that need no mask: every row sees all keys of the tile.
    const uint32_t full_lo = start_of(P.pos0 + tok_last, P);  // max start over the block
    const uint32_t full_hi = P.pos0 + tok0;                   // min position over the block

    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
    const uint64_t row_bytes = (uint64_t)P.kv_heads * 256u;
    const char *kg = reinterpret_cast<const char *>(P.k) + kvh * 256u;
    const char *vg = reinterpret_cast<const char *>(P.v) + kvh * 256u;

    auto issue = [&](uint32_t it) {
        if (it < ntiles) {
            const uint32_t k0 = kbeg + it * kKeys;
            const uint32_t st = sbase + (it % kStages) * 2u * kTileBytes;
            // 64 rows x 16 chunks = 1024 chunks per tensor; NW*32 threads.
            for (uint32_t c = threadIdx.x; c < 1024u; c += NW * 32u) {
                const uint32_t r = c >> 4, ch = c & 15u;
                uint32_t kp = k0 + r;
                if (kp >= kend) kp = kbeg;  // clamp: masked anyway
                const uint64_t go = (uint64_t)(kp % P.cap) * row_bytes + ch * 16u;
                const uint32_t so = r * 256u + ((ch ^ (r & 7u)) << 4);
                cp16(st + so, kg + go);
                cp16(st + kTileBytes + so, vg + go);
            }
        }
        asm volatile("cp.async.commit_group;");
    };

    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

#pragma unroll
    for (int s = 0; s < kStages - 1; s++) issue(s);

    for (uint32_t it = 0; it < ntiles; it++) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 2));
        __syncthreads();
        issue(it + kStages - 1);
        const uint32_t k0 = kbeg + it * kKeys;
        const uint32_t kt = sbase + (it % kStages) * 2u * kTileBytes;
        const uint32_t vt = kt + kTileBytes;

        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {  // pairs of key n-tiles
                const uint32_t r = np * 16u + ((lane >> 4) << 3) + (lane & 7u);
                const uint32_t ch = 2u * kk + ((lane >> 3) & 1u);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kt + r * 256u + ((ch ^ (r & 7u)) << 4), b0, b1, b2, b3);
                mma(s[2 * np], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                mma(s[2 * np + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        }
        const bool need_mask = !(k0 >= full_lo && k0 + kKeys - 1u <= full_hi);
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 8; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int rr = e >> 1;
                float v = s[n][e] * P.qscale;
                if (need_mask) {
                    const uint32_t kp = k0 + n * 8u + 2u * t + (e & 1);
                    if (kp < srow[rr] || kp > prow[rr] || kp >= kend) v = -INFINITY;
                }
                s[n][e] = v;
                mx[rr] = fmaxf(mx[rr], v);
            }
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
        }
        const bool up = (mx[0] > m[0] + 8.f) || (mx[1] > m[1] + 8.f);
        if (__any_sync(0xffffffffu, up)) {
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const float mn = fmaxf(m[rr], mx[rr]);
                const float alpha = mn == -INFINITY ? 1.f : fast_exp2(m[rr] - mn);
                l[rr] *= alpha;
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    o[i][2 * rr] *= alpha;
                    o[i][2 * rr + 1] *= alpha;
                }
                m[rr] = mn;
            }
        }
        const float mu[2] = {m[0] == -INFINITY ? 0.f : m[0], m[1] == -INFINITY ? 0.f : m[1]};
        uint32_t pa[4][4];
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const float p0 = fast_exp2(s[n][0] - mu[0]), p1 = fast_exp2(s[n][1] - mu[0]);
            const float p2 = fast_exp2(s[n][2] - mu[1]), p3 = fast_exp2(s[n][3] - mu[1]);
            l[0] += p0 + p1;
            l[1] += p2 + p3;
            const int kk2 = n >> 1, hi = n & 1;
            pa[kk2][hi ? 2 : 0] = pack_h2(p0, p1);
            pa[kk2][hi ? 3 : 1] = pack_h2(p2, p3);
        }
#pragma unroll
        for (int kk2 = 0; kk2 < 4; kk2++) {
#pragma unroll
            for (int jp = 0; jp < 8; jp++) {  // pairs of dim n-tiles
                const uint32_t r = kk2 * 16u + (((lane >> 3) & 1u) << 3) + (lane & 7u);
                const uint32_t ch = 2u * jp + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vt + r * 256u + ((ch ^ (r & 7u)) << 4), b0, b1, b2, b3);
                mma(o[2 * jp], pa[kk2][0], pa[kk2][1], pa[kk2][2], pa[kk2][3], b0, b1);
                mma(o[2 * jp + 1], pa[kk2][0], pa[kk2][1], pa[kk2][2], pa[kk2][3], b2, b3);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;");

#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
        l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
        const uint32_t tok = tok0 + g + 8u * rr;
        if (tok >= P.n_tok) continue;
        const float gt = P.gate ? sigmoid_dev(P.gate[(uint64_t)tok * P.q_heads + h]) : 1.f;
        const float f = l[rr] > 0.f ? gt / l[rr] : 0.f;
        float *op = P.out + ((uint64_t)tok * P.q_heads + h) * 128u;
#pragma unroll
        for (int n = 0; n < 16; n++)
            *reinterpret_cast<float2 *>(op + n * 8 + 2 * t) = make_float2(o[n][2 * rr] * f, o[n][2 * rr + 1] * f);
    }
}

// ------------------------------------------------------------ f32 caches
// The reference's own cache type (fp32 K/V, fp32 q): the drop-in
// sf37_cuda_attention_prefill_heads.  Same tiling as prefill_mma_kernel (one
// CTA per (16-token block, KV head), one warp per query head), with bf16
// tensor-core tiles in a three-term split: every fp32 operand x is carried
// as hi = rn_bf16(x) and lo = rn_bf16(x - hi) (16 significant bits), and
//   S = Qhi.Khi + Qlo.Khi + Qhi.Klo,   O += Phi.Vhi + Plo.Vhi + Phi.Vlo
// (the dropped lo.lo term is below 2^-16 relative), fp32 accumulate.
// Key tiles of 64 rows stream as fp32 through a 2-stage cp.async ring
// (64 KB per stage); once a tile has landed the CTA converts it once into
// hi/lo bf16 tiles (ldmatrix layout, chunk ^ (row & 7) swizzle) that all G
// warps share.
struct PrefillParams32 {
    const float *k, *v;
    const float *q;     // [n_tok][q_heads][128]
    const float *gate;  // [n_tok][q_heads] or nullptr
    float *out;         // [n_tok][q_heads][128]
    uint32_t pos0, n_tok, cap, sliding, window;
    uint32_t q_heads, kv_heads;
    float qscale;       // log2(e)/sqrt(128)
};

namespace {

constexpr uint32_t kTile32 = kKeys * 512;     // one fp32 tile (K or V)
constexpr uint32_t kStage32 = 2 * kTile32;    // K then V
constexpr uint32_t kConv = kKeys * 256;       // one bf16 tile
constexpr int kStages32 = 2;
constexpr size_t kSmem32 = (size_t)kStages32 * kStage32 + 4 * kConv;

__device__ __forceinline__ void mma_bf(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (hi, lo) bf16x2 of two floats
__device__ __forceinline__ void split_bf2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
__device__ __forceinline__ uint32_t start_of32(uint32_t p, const PrefillParams32 &P) {
    const uint32_t have = p + 1u;
    uint32_t s = have > P.cap ? have - P.cap : 0u;
    if (P.sliding && have > P.window && have - P.window > s) s = have - P.window;
    return s;
}

}  // namespace

template <int NW>
__global__ void __launch_bounds__(NW * 32, 1) prefill_f32_kernel(const __grid_constant__ PrefillParams32 P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t nblk = (P.n_tok + 15u) >> 4;
    const uint32_t tb = nblk - 1u - blockIdx.x;  // longest causal ranges first
    const uint32_t kvh = blockIdx.y;
    const uint32_t h = kvh * NW + warp;           // query head of this warp
    const uint32_t tok0 = tb * 16u;
    const uint32_t tok_last = min(tok0 + 15u, P.n_tok - 1u);

    // Q fragments, scaled by log2(e)/sqrt(d), as hi and lo bf16.
    uint32_t qh[8][4], ql[8][4];
    {
        const uint32_t r0 = min(tok0 + g, P.n_tok - 1u), r1 = min(tok0 + g + 8u, P.n_tok - 1u);
        const float *q0 = P.q + ((uint64_t)r0 * P.q_heads + h) * 128u;
        const float *q1 = P.q + ((uint64_t)r1 * P.q_heads + h) * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            const float2 a0 = *reinterpret_cast<const float2 *>(q0 + kk * 16 + 2 * t);
            const float2 a1 = *reinterpret_cast<const float2 *>(q1 + kk * 16 + 2 * t);
            const float2 a2 = *reinterpret_cast<const float2 *>(q0 + kk * 16 + 8 + 2 * t);
            const float2 a3 = *reinterpret_cast<const float2 *>(q1 + kk * 16 + 8 + 2 * t);
            split_bf2(a0.x * P.qscale, a0.y * P.qscale, qh[kk][0], ql[kk][0]);
            split_bf2(a1.x * P.qscale, a1.y * P.qscale, qh[kk][1], ql[kk][1]);
            split_bf2(a2.x * P.qscale, a2.y * P.qscale, qh[kk][2], ql[kk][2]);
            split_bf2(a3.x * P.qscale, a3.y * P.qscale, qh[kk][3], ql[kk][3]);
        }
    }
    const uint32_t prow[2] = {P.pos0 + tok0 + g, P.pos0 + tok0 + g + 8u};
    const uint32_t srow[2] = {start_of32(prow[0], P), start_of32(prow[1], P)};
    const uint32_t kbeg = start_of32(P.pos0 + tok0, P);
    const uint32_t kend = P.pos0 + tok_last + 1u;
    const uint32_t ntiles = (kend - kbeg + kKeys - 1) / kKeys;
    const uint32_t full_lo = start_of32(P.pos0 + tok_last, P);
    const uint32_t full_hi = P.pos0 + tok0;

    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
    const uint32_t cbase = sbase + kStages32 * kStage32;  // Khi, Klo, Vhi, Vlo
    const uint64_t row_bytes = (uint64_t)P.kv_heads * 512u;
    const char *kg = reinterpret_cast<const char *>(P.k) + kvh * 512u;
    const char *vg = reinterpret_cast<const char *>(P.v) + kvh * 512u;

    auto issue = [&](uint32_t it) {
        if (it < ntiles) {
            const uint32_t k0 = kbeg + it * kKeys;
            const uint32_t st = sbase + (it % kStages32) * kStage32;
            // 64 rows x 32 chunks of 16 B per tensor
            for (uint32_t c = threadIdx.x; c < 2048u; c += NW * 32u) {
                const uint32_t r = c >> 5, ch = c & 31u;
                uint32_t kp = k0 + r;
                if (kp >= kend) kp = kbeg;  // clamp: masked anyway
                const uint64_t go = (uint64_t)(kp % P.cap) * row_bytes + ch * 16u;
                cp16(st + r * 512u + ch * 16u, kg + go);
                cp16(st + kTile32 + r * 512u + ch * 16u, vg + go);
            }
        }
        asm volatile("cp.async.commit_group;");
    };

    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

#pragma unroll
    for (int s = 0; s < kStages32; s++) issue(s);

    for (uint32_t it = 0; it < ntiles; it++) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kStages32 - 1));
        __syncthreads();  // stage it landed; the previous tile's bf16 tiles are no longer read
        {
            // fp32 stage -> hi / lo bf16 tiles: a thread converts 8 floats
            // (one 16-byte bf16 chunk) of K or V per step.
            const uint8_t *st = smem + (it % kStages32) * kStage32;
            for (uint32_t c = threadIdx.x; c < 2048u; c += NW * 32u) {
                const uint32_t tsr = c >> 10, r = (c >> 4) & 63u, ch = c & 15u;  // tensor, row, bf16 chunk
                const float4 x0 = *reinterpret_cast<const float4 *>(st + tsr * kTile32 + r * 512u + ch * 32u);
                const float4 x1 = *reinterpret_cast<const float4 *>(st + tsr * kTile32 + r * 512u + ch * 32u + 16u);
                uint4 hi, lo;
                split_bf2(x0.x, x0.y, hi.x, lo.x);
                split_bf2(x0.z, x0.w, hi.y, lo.y);
                split_bf2(x1.x, x1.y, hi.z, lo.z);
                split_bf2(x1.z, x1.w, hi.w, lo.w);
                const uint32_t so = r * 256u + ((ch ^ (r & 7u)) << 4);
                uint8_t *cb = smem + kStages32 * kStage32 + tsr * 2u * kConv;
                *reinterpret_cast<uint4 *>(cb + so) = hi;
                *reinterpret_cast<uint4 *>(cb + kConv + so) = lo;
            }
        }
        __syncthreads();  // bf16 tiles ready; stage it is free
        issue(it + kStages32);
        const uint32_t k0 = kbeg + it * kKeys;
        const uint32_t khi = cbase, klo = cbase + kConv, vhi = cbase + 2u * kConv, vlo = cbase + 3u * kConv;

        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {
                const uint32_t r = np * 16u + ((lane >> 4) << 3) + (lane & 7u);
                const uint32_t ch = 2u * kk + ((lane >> 3) & 1u);
                const uint32_t off = r * 256u + ((ch ^ (r & 7u)) << 4);
                uint32_t b0, b1, b2, b3, c0, c1, c2, c3;
                ldsm_x4(khi + off, b0, b1, b2, b3);
                ldsm_x4(klo + off, c0, c1, c2, c3);
                mma_bf(s[2 * np], qh[kk], b0, b1);
                mma_bf(s[2 * np], ql[kk], b0, b1);
                mma_bf(s[2 * np], qh[kk], c0, c1);
                mma_bf(s[2 * np + 1], qh[kk], b2, b3);
                mma_bf(s[2 * np + 1], ql[kk], b2, b3);
                mma_bf(s[2 * np + 1], qh[kk], c2, c3);
            }
        }
        const bool need_mask = !(k0 >= full_lo && k0 + kKeys - 1u <= full_hi);
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 8; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int rr = e >> 1;
                float v = s[n][e];
                if (need_mask) {
                    const uint32_t kp = k0 + n * 8u + 2u * t + (e & 1);
                    if (kp < srow[rr] || kp > prow[rr] || kp >= kend) v = -INFINITY;
                }
                s[n][e] = v;
                mx[rr] = fmaxf(mx[rr], v);
            }
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
        }
        const bool up = (mx[0] > m[0] + 8.f) || (mx[1] > m[1] + 8.f);
        if (__any_sync(0xffffffffu, up)) {
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const float mn = fmaxf(m[rr], mx[rr]);
                const float alpha = mn == -INFINITY ? 1.f : exp2f(m[rr] - mn);
                l[rr] *= alpha;
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    o[i][2 * rr] *= alpha;
                    o[i][2 * rr + 1] *= alpha;
                }
                m[rr] = mn;
            }
        }
        const float mu[2] = {m[0] == -INFINITY ? 0.f : m[0], m[1] == -INFINITY ? 0.f : m[1]};
        uint32_t ph[4][4], pl[4][4];
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const float p0 = exp2f(s[n][0] - mu[0]), p1 = exp2f(s[n][1] - mu[0]);
            const float p2 = exp2f(s[n][2] - mu[1]), p3 = exp2f(s[n][3] - mu[1]);
            l[0] += p0 + p1;
            l[1] += p2 + p3;
            const int kk2 = n >> 1, hi = n & 1;
            split_bf2(p0, p1, ph[kk2][hi ? 2 : 0], pl[kk2][hi ? 2 : 0]);
            split_bf2(p2, p3, ph[kk2][hi ? 3 : 1], pl[kk2][hi ? 3 : 1]);
        }
#pragma unroll
        for (int kk2 = 0; kk2 < 4; kk2++) {
#pragma unroll
            for (int jp = 0; jp < 8; jp++) {
                const uint32_t r = kk2 * 16u + (((lane >> 3) & 1u) << 3) + (lane & 7u);
                const uint32_t ch = 2u * jp + (lane >> 4);
                const uint32_t off = r * 256u + ((ch ^ (r & 7u)) << 4);
                uint32_t b0, b1, b2, b3, c0, c1, c2, c3;
                ldsm_x4_t(vhi + off, b0, b1, b2, b3);
                ldsm_x4_t(vlo + off, c0, c1, c2, c3);
                mma_bf(o[2 * jp], ph[kk2], b0, b1);
                mma_bf(o[2 * jp], pl[kk2], b0, b1);
                mma_bf(o[2 * jp], ph[kk2], c0, c1);
                mma_bf(o[2 * jp + 1], ph[kk2], b2, b3);
                mma_bf(o[2 * jp + 1], pl[kk2], b2, b3);
                mma_bf(o[2 * jp + 1], ph[kk2], c2, c3);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;");

#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
        l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
        const uint32_t tok = tok0 + g + 8u * rr;
        if (tok >= P.n_tok) continue;
        const float gt = P.gate ? sigmoid_dev(P.gate[(uint64_t)tok * P.q_heads + h]) : 1.f;
        const float f = l[rr] > 0.f ? gt / l[rr] : 0.f;
        float *op = P.out + ((uint64_t)tok * P.q_heads + h) * 128u;
#pragma unroll
        for (int n = 0; n < 16; n++)
            *reinterpret_cast<float2 *>(op + n * 8 + 2 * t) = make_float2(o[n][2 * rr] * f, o[n][2 * rr + 1] * f);
    }
}

// fp32 caches and fp32 queries on tensor cores (group 4 or 8, head_dim 128,
// 16-byte aligned buffers); *handled stays false for other shapes.
int prefill_tc32(const sf37kv_cache *cache, const float *q, const float *gate, float *out, uint32_t pos0,
                 uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads, cudaStream_t stream, bool *handled) {
    *handled = false;
    if (kv_heads == 0 || q_heads % kv_heads) return SF37KV_OK;
    const uint32_t G = q_heads / kv_heads;
    if (G != 4 && G != 8) return SF37KV_OK;
    if (((uintptr_t)cache->k_cache | (uintptr_t)cache->v_cache | (uintptr_t)q) & 15u) return SF37KV_OK;
    if ((uint64_t)pos0 + n_tok > 0xffffffffull) return set_error(SF37KV_EINVAL, "prefill: positions overflow");
    PrefillParams32 P{(const float *)cache->k_cache, (const float *)cache->v_cache, q, gate, out, pos0, n_tok,
                      cache->cap, cache->sliding, cache->window, q_heads, kv_heads,
                      1.4426950408889634f / sqrtf(128.0f)};
    dim3 grid((n_tok + 15) / 16, kv_heads);
    if (G == 4) {
        cudaFuncSetAttribute(prefill_f32_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem32);
        prefill_f32_kernel<4><<<grid, 128, kSmem32, stream>>>(P);
    } else {
        cudaFuncSetAttribute(prefill_f32_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem32);
        prefill_f32_kernel<8><<<grid, 256, kSmem32, stream>>>(P);
    }
    g_launches++;
    if (int rc = check_cuda(cudaGetLastError(), "prefill f32 tensor-core launch")) return rc;
    *handled = true;
    return SF37KV_OK;
}

int prefill_tc(const sf37kv_cache *cache, const void *q, int q_type, const float *gate, float *out,
               uint32_t pos0, uint32_t n_tok, uint32_t q_heads, uint32_t kv_heads, cudaStream_t stream,
               bool *handled) {
    *handled = false;
    if (q_type != SF37KV_Q_BF16 || kv_heads == 0 || q_heads % kv_heads) return SF37KV_OK;
    const uint32_t G = q_heads / kv_heads;
    if (G != 4 && G != 8 && G != 12 && G != 16) return SF37KV_OK;
    if (((uintptr_t)cache->k_cache | (uintptr_t)cache->v_cache | (uintptr_t)q) & 15u) return SF37KV_OK;
    if ((uint64_t)pos0 + n_tok > 0xffffffffull) return set_error(SF37KV_EINVAL, "prefill: positions overflow");
    PrefillParams P{(const __half *)cache->k_cache, (const __half *)cache->v_cache, (const uint16_t *)q, gate,
                    out, pos0, n_tok, cache->cap, cache->sliding, cache->window, q_heads, kv_heads,
                    1.4426950408889634f / sqrtf(128.0f)};
    const size_t sm = (size_t)kStages * 2 * kTileBytes;
    dim3 grid((n_tok + 15) / 16, kv_heads);
#define SF37_PF(NWV)                                                                                       \
    do {                                                                                                   \
        cudaFuncSetAttribute(prefill_mma_kernel<NWV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm); \
        prefill_mma_kernel<NWV><<<grid, NWV * 32, sm, stream>>>(P);                                         \
    } while (0)
    switch (G) {
        case 4: SF37_PF(4); break;
        case 8: SF37_PF(8); break;
        case 12: SF37_PF(12); break;
        default: SF37_PF(16); break;
    }
#undef SF37_PF
    g_launches++;
    if (int rc = check_cuda(cudaGetLastError(), "prefill tensor-core launch")) return rc;
    *handled = true;
    return SF37KV_OK;
}

}  // namespace sf37kv
