// GQA decode attention over ring-indexed KV caches: split-K flash-decoding.
//
// Semantics (reference sf37_cuda.cu:2384-3161): for query head h of KV head
// kvh = h / G (G = q_heads / kv_heads), over logical rows [start, end) at ring
// slot r % cap:  out[h] = softmax(q[h].K[r] / sqrt(d)) . V[r] * sigmoid(gate[h]).
//
// Work decomposition (all kernels): one CTA per (job, kv head, split), where
// a job is one layer's query (decode) or one prefill token (fallback path)
// and a split is a contiguous run of rows.  Every CTA serves all G query
// heads of its KV head, so each K/V byte is read from HBM once per group.
// Inside a CTA the warps take interleaved 16-row (f16) or 4/8-row (f32)
// blocks, keep an online softmax state each, and merge through shared memory.
// With more than one split per (job, kv head), each CTA writes a partial
// (O, max, sum) to scratch; the last CTA to finish (atomic counter) merges
// the partials and writes the output, so a whole multi-layer step is one
// launch.  Scores are kept in the log2 domain (q pre-scaled by
// log2(e)/sqrt(d)); a running max is only raised when a block's max exceeds
// it by more than 8 (2^8 headroom), which removes almost all O rescaling.
//
// f16 caches (the throughput path, head_dim 128, G <= 16): QK^T and PV are
// mma.sync m16n8k16 tiles fed straight from 128-bit global loads in
// registers (no shared-memory staging: the dimension order inside a head is
// permuted so each thread's loaded words already are its mma fragments).
// The 16 M-rows of a tile hold 8 query heads twice: rows 0-7 carry the f16
// "hi" part of q (and of P), rows 8-15 the f16 remainder "lo", so q.K and
// P.V are computed to ~22 mantissa bits with fp32 accumulation at no extra
// mma cost.  This is a bandwidth-bound gather; the tensor cores only keep the
// FMA count out of the way.
//
// f32 caches (the reference-compatible path): CUDA-core fp32 kernel, lanes
// over the head dimension, partial dot products of several rows x heads
// reduced with a transposing butterfly (N values over 32 lanes in N-1
// shuffles).
//
// Anything else (head_dim != 128, other G): a generic warp-per-head kernel.
#include <cfloat>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <mutex>

#include <cuda_bf16.h>
#include <cmath>

#include "kv_internal.cuh"
#include "../../include/sf37_cuda_kv.h"

namespace sf37kv {

extern unsigned long long g_launches;

constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kMaxSplits = 256;
constexpr float kRescaleSlack = 8.0f;

// Set by attention_jobs_gather for the duration of one attention_jobs call.
static const GatherDev *g_gather_cur = nullptr;
static uint64_t g_gather_off[kMaxJobs];

struct JobDev {
    const void *k;
    const void *v;
    const float *q;
    const float *gate;
    float *out;
    uint32_t start, end, cap;
    uint32_t split_rows, n_splits, cta_begin;
    const float *k_new, *v_new;  // appended row (position end-1) or nullptr
    uint64_t gather_off;         // float offset of this job's block in the peers' gather buffers
    // q/k head preparation (qn == nullptr: none): RMS norm with weight
    // (w + 1) then split-half RoPE over `rotary` dims with the cos/sin table
    // DecodeParams::rope[rope_idx].
    const uint16_t *qn, *kn;     // bf16 [128] norm weights
    uint32_t rotary, rope_idx;
    float eps;
    uint32_t pre;                // rows may be streamed before griddepcontrol.wait
};

// RoPE cos/sin tables of one decode launch: one per distinct (rotary_dim,
// theta, llama3, position), cos of pairs 0..63 then sin.  Computed on the
// host with the reference's own arithmetic (see rope_table below).
constexpr int kMaxRope = 8;

// The G query heads of KV head kvh (and, with_k, the new K row's head kvh)
// normalized and rotated into shared memory Qf [G][128] / Kf [128]:
//   head_rms_norm_weight1 (sf37.c:1921-1929 -> sf37_rms_norm_weight1,
//   sf37_ops.c:22-28: double sum of squares, scale = 1 / sqrtf(mean + eps),
//   x * scale * (w + 1)), then apply_rope_one (sf37.c:2015-2031): pairs
//   (i, i + rotary/2) rotated by the host-made cos/sin table `rope`.
// One warp per head; every warp of the CTA takes part.
__device__ __noinline__ void prep_heads(const float *rope, const JobDev &J, uint32_t kvh, uint32_t G,
                                        bool with_k, float *Qf, float *Kf) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint32_t half = J.rotary >> 1;
    const uint32_t nh = G + (with_k ? 1u : 0u);
    // Issue every global load first (heads warp, warp + nw, ...; at most 5
    // per warp for G <= 16 and 4 warps), then compute.
    constexpr int kR = 5;
    float4 xs[kR];
#pragma unroll
    for (int r = 0; r < kR; r++) {
        const uint32_t h = warp + (uint32_t)r * nw;
        xs[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (h < nh) {
            const float *src = h == G ? J.k_new + kvh * 128u : J.q + (uint64_t)(kvh * G + h) * 128u;
            xs[r] = reinterpret_cast<const float4 *>(src)[lane];
        }
    }
    const uint2 wq = reinterpret_cast<const uint2 *>(J.qn)[lane];
    const uint2 wk = with_k ? reinterpret_cast<const uint2 *>(J.kn)[lane] : make_uint2(0u, 0u);
    float cs[2], sn[2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const uint32_t i = lane + 32u * u;
        cs[u] = i < half ? rope[i] : 1.f;
        sn[u] = i < half ? rope[64u + i] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < kR; r++) {
        const uint32_t h = warp + (uint32_t)r * nw;
        if (h >= nh) break;
        const bool isk = h == G;
        const float4 x = xs[r];
        const uint2 wb = isk ? wk : wq;
        float *dst = isk ? Kf : Qf + h * 128u;
        double ss = (double)x.x * x.x + (double)x.y * x.y + (double)x.z * x.z + (double)x.w * x.w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float scale = 1.0f / sqrtf((float)(ss / 128.0) + J.eps);
        const float w0 = __uint_as_float(wb.x << 16) + 1.0f, w1 = __uint_as_float(wb.x & 0xffff0000u) + 1.0f;
        const float w2 = __uint_as_float(wb.y << 16) + 1.0f, w3 = __uint_as_float(wb.y & 0xffff0000u) + 1.0f;
        reinterpret_cast<float4 *>(dst)[lane] =
            make_float4(x.x * scale * w0, x.y * scale * w1, x.z * scale * w2, x.w * scale * w3);
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const uint32_t i = lane + 32u * u;
            if (i < half) {
                const float a = dst[i], b = dst[i + half];
                dst[i] = a * cs[u] - b * sn[u];
                dst[i + half] = b * cs[u] + a * sn[u];
            }
        }
        __syncwarp();
    }
}

// The CTA whose rows end at the job's last row (end-1) stores this KV head's
// slice of the appended row (f32 -> T, round to nearest even) before any warp loads
// rows; __syncthreads() plus L2-coherent cp.async.cg loads make it visible.
template <typename T>
__device__ __forceinline__ void fused_append(const JobDev &J, uint32_t kvh, bool appender, uint32_t kv_heads,
                                             const float *kf = nullptr) {
    if (!appender) return;
    const uint32_t i = threadIdx.x;
    if (i >= 64u) return;
    // kf: the prepared K head in shared memory (prep_heads), else the raw row
    const float *src = i < 32u ? (kf ? kf + (i & 31u) * 4u : J.k_new + kvh * 128u + (i & 31u) * 4u)
                               : J.v_new + kvh * 128u + (i & 31u) * 4u;
    const float4 x = *reinterpret_cast<const float4 *>(src);
    T *dst = reinterpret_cast<T *>(const_cast<void *>(i < 32u ? J.k : J.v)) +
             (uint64_t)((J.end - 1u) % J.cap) * kv_heads * 128u + kvh * 128u + (i & 31u) * 4u;
    if (sizeof(T) == 4) {
        *reinterpret_cast<float4 *>(dst) = x;
    } else {
        const __half2 a = __floats2half2_rn(x.x, x.y), b = __floats2half2_rn(x.z, x.w);
        *reinterpret_cast<uint2 *>(dst) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
    }
}

struct DecodeParams {
    JobDev job[kMaxJobs];
    uint32_t n_jobs, total_ctas;
    uint32_t q_heads, kv_heads, group;
    uint32_t part_stride;  // floats per CTA partial: G*128 O, then G (m, l) pairs
    float *part;
    uint32_t *counters;    // one per (job, kv head)
    float qscale;          // log2(e) / sqrt(head_dim)
    GatherDev gat;
    float rope[kMaxRope][128];  // q/k preparation tables (JobDev::rope_idx)
    uint32_t pdl;               // launched with programmatic stream serialization
    int *err;                   // device error flag (a bounded wait gave up), or nullptr
};

// Programmatic dependent launch (sm_90+): a kernel launched with
// programmatic stream serialization may start while the previous kernel on
// the stream is still running; griddepcontrol.wait blocks until that kernel
// has completed and its writes are visible.  Without the attribute both are
// no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void gather_store(const DecodeParams &P, const JobDev &J, uint64_t idx, float v) {
    for (uint32_t p = 0; p < P.gat.world; p++)
        if (p != P.gat.rank) P.gat.peer[p][J.gather_off + idx] = v;
}
__device__ __forceinline__ void gather_store4(const DecodeParams &P, const JobDev &J, uint64_t idx, float4 v) {
    for (uint32_t p = 0; p < P.gat.world; p++)
        if (p != P.gat.rank) *reinterpret_cast<float4 *>(P.gat.peer[p] + J.gather_off + idx) = v;
}
// Called by every CTA that wrote final outputs of one (job, kv head) group.
// Thread 0's system-scope acq_rel atomic publishes the CTA's peer stores
// (they precede it through the barrier); the last group's acquire has seen
// every group's, and one system fence then releases all flag stores at once
// (a release store per peer would pay a fence per peer).  Measured at 8
// GPUs: gather launch 145 -> 140 us with the atomic in place of a system
// fence per group.
__device__ __forceinline__ void gather_group_done(const DecodeParams &P) {
    if (!P.gat.world) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t prev;
        asm volatile("atom.acq_rel.sys.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(P.gat.done) : "memory");
        if (prev == P.gat.total_groups - 1u) {
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            for (uint32_t p = 0; p < P.gat.world; p++) {
                uint32_t *f = P.gat.peer_flags[p] + P.gat.rank;
                asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(P.gat.epoch) : "memory");
            }
            *P.gat.done = 0u;
        }
    }
}

// ------------------------------------------------------------ helpers
__device__ __forceinline__ uint32_t locate_job(const DecodeParams &P, uint32_t cta) {
    uint32_t j = 0;
    while (j + 1 < P.n_jobs && P.job[j + 1].cta_begin <= cta) j++;
    return j;
}

__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

__device__ __forceinline__ float4 ld_stream_f4(const void *p) {
    uint4 r = ld_stream16(p);
    return make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z),
                       __uint_as_float(r.w));
}

__device__ __forceinline__ uint32_t word_of(const uint4 &u, int w) {
    return w == 0 ? u.x : (w == 1 ? u.y : (w == 2 ? u.z : u.w));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Slot of logical row base + x, given sb = base % cap.
__device__ __forceinline__ uint32_t ring_slot(uint32_t sb, uint32_t x, uint32_t cap) {
    uint32_t s = sb + x;
    if (s >= cap) s -= cap;
    if (s >= cap) s %= cap;  // only when cap < 16
    return s;
}

// Streaming copy of K/V rows with an L2 evict-first policy: a decode step
// reads far more K/V than L2 holds, and without the hint the stream evicts
// what the kernel's tail needs hot -- its own instructions, q, the split
// partials and counters -- so every cold access of the epilogue waits behind
// the HBM queue.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void cp_async16_ef(uint32_t smem_addr, const void *gptr, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_addr), "l"(gptr), "l"(pol));
}
__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void *gptr) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gptr));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

// ------------------------------------------------------------ CTA epilogue
// Shared memory used by the epilogue: per stream and head, O[128], m, l.
//   Os[os_at(stream * 16 + h, d)], Ms[stream*16 + h], Ls[stream*16 + h]
// followed by X: W[stream*16 + h] (stream weights), PM[16], PL[16].
// After the stream merge, the CTA's result is written either directly to the
// output (single split) or to scratch followed by the last-CTA reduction.

// Float index of dimension d of row `row` (= stream * 16 + head) in Os: rows
// of 128 floats whose 16-byte chunks are permuted by chunk ^ (row & 7) ^
// ((chunk >> 3) & 3).  The warps' fragment stores (8 heads x 4 column groups
// per instruction) then spread over the banks instead of landing 16- or
// 32-fold on one, and float4 reads of a row stay whole and conflict free.
__device__ __forceinline__ uint32_t os_at(uint32_t row, uint32_t d) {
    const uint32_t c = d >> 2;
    return row * 128u + ((c ^ (row & 7u) ^ ((c >> 3) & 3u)) << 2) + (d & 3u);
}

// Stream weights of each head h < G: M = max over streams of m, W[s][h] =
// 2^(m_s - M), L = sum_s l_s W[s][h].  Warp w takes heads w, w + nw, ...;
// lane s takes stream s (n_streams <= 32), reductions by shuffles.
__device__ __forceinline__ void stream_weights(uint32_t G, uint32_t n_streams, const float *Ms, const float *Ls,
                                               float *W, float *PM, float *PL) {
    const uint32_t lane = threadIdx.x & 31u, nw = blockDim.x >> 5;
    for (uint32_t h = threadIdx.x >> 5; h < G; h += nw) {
        const bool on = lane < n_streams;
        const float m = on ? Ms[lane * 16u + h] : -INFINITY;
        float M = m;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float w = (M == -INFINITY || !on) ? 0.f : fast_exp2(m - M);
        float L = on ? Ls[lane * 16u + h] * w : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (on) W[lane * 16u + h] = w;
        if (lane == 0) {
            PM[h] = M;
            PL[h] = L;
        }
    }
}

// sum_s W[s][h] * O_s[h][d4 .. d4+3]
__device__ __forceinline__ float4 stream_o(uint32_t n_streams, const float *Os, const float *W, uint32_t h,
                                           uint32_t d4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t s = 0; s < n_streams; s++) {
        const float w = W[s * 16u + h];
        const float4 o = *reinterpret_cast<const float4 *>(Os + os_at(s * 16u + h, d4));
        acc.x += o.x * w;
        acc.y += o.y * w;
        acc.z += o.z * w;
        acc.w += o.w * w;
    }
    return acc;
}

__device__ __forceinline__ float4 finalize4(float4 acc, float L, float g) {
    float4 r;
    r.x = L > 0.f ? acc.x / L * g : 0.f;
    r.y = L > 0.f ? acc.y / L * g : 0.f;
    r.z = L > 0.f ? acc.z / L * g : 0.f;
    r.w = L > 0.f ? acc.w / L * g : 0.f;
    return r;
}

__device__ __forceinline__ float *epilogue_x(float *Ls, uint32_t G, uint32_t n_streams) {
    float *X = Ls + 16u * n_streams * ((G + 7u) >> 3);
    return reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(X) + 15u) & ~uintptr_t(15));
}

// Bulk (TMA) copies for the split merge: one transaction per partial,
// completion counted on an mbarrier.  Addresses and sizes are multiples of
// 16 bytes (partials are part_stride floats, part_stride a multiple of 4).
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// Parity wait with an iteration bound (the copies are from this GPU's own
// memory and complete in microseconds; the bound only keeps a fault from
// hanging the kernel).  Returns false when it gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(bar), "r"(phase)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > 4000000000ll) return false;
    }
}

// The last CTA of a (job, KV head) merges its n split partials.  Thread 0
// starts bulk copies of whole partials (O vectors and (m, l) pairs) into the
// stage buffers, as many splits per pass as fit (all of them for the small-
// launch plan), so a pass costs one L2 round trip.  Per pass the weights are
// computed once per (split, head) in parallel -- running max M_h, the old
// state's rescale 2^(M_old - M_h), w[s][h] = 2^(m_s - M_h) -- and each
// thread then folds its float4s of O with independent multiply-adds.
constexpr uint32_t kMergePass = 48;  // splits per pass at most
template <int NT>
__device__ void merge_partials(const DecodeParams &P, const JobDev &J, uint32_t kvh, uint8_t *smem,
                               uint32_t stage_bytes, const float *gate_s) {
    __shared__ float mw[kMergePass * 16];        // w[s][h]
    __shared__ float mM[16], mScale[16], mL[16];  // running max, rescale of the old state, running sum
    const uint32_t G = P.group, n = J.n_splits, stride = P.part_stride, tid = threadIdx.x;
    const float *P0 = P.part + (uint64_t)(J.cta_begin + kvh * n) * stride;
    const uint32_t split_bytes = stride * 4u;
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(smem + stage_bytes - 16u);
    uint32_t cnt_max = (stage_bytes - 16u) / split_bytes;
    if (cnt_max > kMergePass) cnt_max = kMergePass;
    if (cnt_max < 1) cnt_max = 1;
    const uint32_t land = (uint32_t)__cvta_generic_to_shared(smem);
    auto issue = [&](uint32_t s0) {
        const uint32_t cnt = min(cnt_max, n - s0);
        // the landing area was last touched by generic loads and stores
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(bar, cnt * split_bytes);
        for (uint32_t s = 0; s < cnt; s++)
            bulk_g2s(land + s * split_bytes, P0 + (uint64_t)(s0 + s) * stride, split_bytes, bar);
    };
    if (tid == 0) {
        mbar_init(bar, 1);
        // the partials were written by other CTAs' generic stores and are
        // read here by the async proxy
        asm volatile("fence.proxy.async.global;" ::: "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        issue(0);
    }
    if (tid < 16) {
        mM[tid] = -INFINITY;
        mL[tid] = 0.f;
    }
    __syncthreads();
    const float *Lf = reinterpret_cast<const float *>(smem);
    const float4 *L4 = reinterpret_cast<const float4 *>(smem);
    constexpr int kPer = (16 * 32 + NT - 1) / NT;  // float4 outputs per thread (G <= 16)
    float4 acc[kPer];
#pragma unroll
    for (int k = 0; k < kPer; k++) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    bool ok = true;
    uint32_t phase = 0;
    for (uint32_t s0 = 0; s0 < n; s0 += cnt_max) {
        const uint32_t cnt = min(cnt_max, n - s0);
        if (!mbar_wait(bar, phase)) ok = false;
        phase ^= 1u;
        if (ok) {
            // per head (warp w: heads w, w + nw, ...; lanes over the pass's
            // splits): running max, rescale of the old state, split
            // weights and the running sum, all by shuffles
            const uint32_t lane = tid & 31u, nw = NT / 32u;
            for (uint32_t h = tid >> 5; h < G; h += nw) {
                float mp = -INFINITY;
                for (uint32_t s = lane; s < cnt; s += 32u) mp = fmaxf(mp, Lf[s * stride + G * 128u + 2u * h]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, o));
                const float mo = mM[h], mn = fmaxf(mo, mp);
                float L = 0.f;
                for (uint32_t s = lane; s < cnt; s += 32u) {
                    const float w = mn == -INFINITY ? 0.f : fast_exp2(Lf[s * stride + G * 128u + 2u * h] - mn);
                    mw[s * 16u + h] = w;
                    L += Lf[s * stride + G * 128u + 2u * h + 1u] * w;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
                __syncwarp();
                if (lane == 0) {
                    const float sc = mo == -INFINITY ? 0.f : fast_exp2(mo - mn);
                    mScale[h] = sc;
                    mL[h] = mL[h] * sc + L;
                    mM[h] = mn;
                }
            }
            __syncthreads();
#pragma unroll
            for (int k = 0; k < kPer; k++) {
                const uint32_t idx = tid + (uint32_t)k * NT;
                if (idx >= G * 32u) continue;
                const uint32_t h = idx >> 5;
                const float sc = mScale[h];
                float4 a = make_float4(acc[k].x * sc, acc[k].y * sc, acc[k].z * sc, acc[k].w * sc);
#pragma unroll 4
                for (uint32_t s = 0; s < cnt; s++) {
                    const float w = mw[s * 16u + h];
                    const float4 v = L4[s * (stride / 4u) + idx];
                    a.x = fmaf(v.x, w, a.x);
                    a.y = fmaf(v.y, w, a.y);
                    a.z = fmaf(v.z, w, a.z);
                    a.w = fmaf(v.w, w, a.w);
                }
                acc[k] = a;
            }
        }
        __syncthreads();
        if (s0 + cnt_max < n && tid == 0 && ok) issue(s0 + cnt_max);
    }
    if (!ok) {
        if (tid == 0 && P.err) atomicExch(P.err, 3);
        return;
    }
#pragma unroll
    for (int k = 0; k < kPer; k++) {
        const uint32_t idx = tid + (uint32_t)k * NT;
        if (idx < G * 32u) {
            const uint32_t h = idx >> 5, d4 = (idx & 31u) * 4u;
            const uint32_t qh = kvh * G + h;
            const float4 r = finalize4(acc[k], mL[h], gate_s[h]);
            *reinterpret_cast<float4 *>(J.out + (uint64_t)qh * 128u + d4) = r;
            if (P.gat.world) gather_store4(P, J, (uint64_t)qh * 128u + d4, r);
        }
    }
}

template <int NT>
__device__ void finish_cta(const DecodeParams &P, const JobDev &J, uint32_t j, uint32_t kvh,
                           uint32_t split, uint32_t cta, uint32_t n_streams, float *Os, float *Ms,
                           float *Ls, uint8_t *smem, uint32_t stage_bytes, const float *gate_s) {
    const uint32_t G = P.group;
    const uint32_t tid = threadIdx.x;
    float *W = epilogue_x(Ls, G, n_streams), *PM = W + 256, *PL = PM + 16;
    __syncthreads();
    stream_weights(G, n_streams, Ms, Ls, W, PM, PL);
    __syncthreads();
    const bool single = J.n_splits == 1;
    float *part = P.part + (uint64_t)cta * P.part_stride;
    for (uint32_t idx = tid; idx < G * 32u; idx += NT) {
        const uint32_t h = idx >> 5, d4 = (idx & 31u) * 4u;
        const float4 acc = stream_o(n_streams, Os, W, h, d4);
        if (single) {
            const uint32_t qh = kvh * G + h;
            const float4 r = finalize4(acc, PL[h], gate_s[h]);
            *reinterpret_cast<float4 *>(J.out + (uint64_t)qh * 128u + d4) = r;
            if (P.gat.world) gather_store4(P, J, (uint64_t)qh * 128u + d4, r);
        } else {
            __stcg(reinterpret_cast<float4 *>(part + h * 128u + d4), acc);
        }
    }
    if (single) {
        gather_group_done(P);
        return;
    }
    if (tid < G) __stcg(reinterpret_cast<float2 *>(part + G * 128u + 2u * tid), make_float2(PM[tid], PL[tid]));

    // Last-CTA election: every thread's partial stores precede the barrier;
    // thread 0's release atomic publishes them (the grid-barrier pattern),
    // and its acquire side orders the merging CTA's reads after the others'.
    __shared__ uint32_t s_last;
    __syncthreads();
    uint32_t *ctr = P.counters + (uint64_t)j * P.kv_heads + kvh;
    if (tid == 0) {
        uint32_t prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ctr) : "memory");
        s_last = prev == J.n_splits - 1u;
    }
    __syncthreads();
    if (!s_last) return;
    // (thread 0's acquire above orders the bulk copies it issues next)
    merge_partials<NT>(P, J, kvh, smem, stage_bytes, gate_s);
    if (tid == 0) *ctr = 0u;  // ready for the next launch
    gather_group_done(P);
}

// ------------------------------------------------------------ f16 kernel: register fragments
// NW warps; warp w handles M-tile (w % n_mt) (query heads 8*mt .. 8*mt+7 of
// the group) and row stream (w / n_mt).  Thread (g = lane/4, t = lane%4).
//
// Register fragments (mma m16n8k16, A row-major 16x16, B col-major 16x8):
//  * QK^T: B[k][n] = K[row b+8i+n][pi(k)], the head dimension permuted so
//    that thread (g,t) holds 16-byte chunks t, t+4, t+8, t+12 of row b+8i+g;
//    the 16 words of those chunks are, in order, the B registers of the 8
//    k-steps.  A = q in the same permutation: row g = hi(q[head g]), row
//    g+8 = lo(q[head g]).  S = C[row g] + C[row g+8].
//  * PV: A = P from the S accumulators (FlashAttention-2 register reuse),
//    rows g / g+8 = hi / lo of p.  B[k][n] = V[row b+k][sigma(n-tile, n)]:
//    thread (g,t) loads rows b+2t, b+2t+1, b+2t+8, b+2t+9, chunks g and g+8,
//    and interleaves the two rows of each B register with one PRMT.
//    Output dim of (n-tile jt, column c) = jt<8 ? 8c+jt : 64+8c+jt-8.
// ------------------------------------------------------------ f16 kernel, cp.async pipeline
// The math and register fragments above; K/V blocks are
// staged through a per-warp ring of S shared-memory stages filled with
// 16-byte cp.async copies, so S-1 blocks (8 KB each) per warp are in flight
// without holding registers.  Warps never wait on each other inside the
// loop (per-warp cp.async groups + __syncwarp).
//
// Stage layout: K tile then V tile, each [16 rows][16 chunks of 16 B]; chunk
// ch of row r sits at slot ch ^ swz(r), swz(r) = ((r&1)<<2) ^ (((r>>1)&3)<<1),
// which makes both fragment read patterns (K: rows g/g+8, chunks 4c+t; V:
// rows 2t+{0,1,8,9}, chunks g/g+8) bank-conflict free for 128-bit loads.
__device__ __forceinline__ uint32_t swz(uint32_t r) { return ((r & 1u) << 2) ^ (((r >> 1) & 3u) << 1); }


__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}

template <int NW, int S, bool PREP = false>
__global__ void __launch_bounds__(NW * 32, 1) decode_f16_pipe_kernel(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    constexpr uint32_t kStage = 8192;  // 16 rows x 256 B for K, then V
    uint4 *Qs = reinterpret_cast<uint4 *>(smem_raw + NW * S * kStage);  // [n_mt][8 kk][32 lanes]
    // Epilogue arrays alias the stage buffers once the loop is done.
    float *Os = reinterpret_cast<float *>(smem_raw);
    float *Ms = Os + NW * 16 * 128;
    float *Ls = Ms + 16 * NW;

    const uint32_t cta = blockIdx.x;
    const uint32_t j = locate_job(P, cta);
    const JobDev &J = P.job[j];
    const uint32_t local = cta - J.cta_begin;
    const uint32_t kvh = local / J.n_splits, split = local - kvh * J.n_splits;
    const uint32_t G = P.group;
    const uint32_t n_mt = (G + 7u) >> 3;
    const uint32_t n_streams = NW / n_mt;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t mt = warp % n_mt, stream = warp / n_mt;

    const uint32_t row0 = J.start + split * J.split_rows;
    const uint32_t row1 = min(row0 + J.split_rows, J.end);
    const uint32_t cap = J.cap;
    const uint64_t row_bytes = (uint64_t)P.kv_heads * 256u;
    const char *kbase = reinterpret_cast<const char *>(J.k) + kvh * 256u;
    const char *vbase = reinterpret_cast<const char *>(J.v) + kvh * 256u;
    const uint32_t qs_addr = (uint32_t)__cvta_generic_to_shared(Qs + mt * 8 * 32 + lane);
    const uint32_t wbuf = (uint32_t)__cvta_generic_to_shared(smem_raw) + warp * S * kStage;

    const uint32_t bstep = n_streams * 16u;
    const uint32_t b_first = row0 + stream * 16u;
    const uint32_t nblk = b_first < row1 ? (row1 - b_first + bstep - 1) / bstep : 0u;

    // Copy block `it` (rows b_first + it*bstep ...) into stage it % S.
    // Lane copies chunks c = lane + 32*i (i < 8) of K and of V: row c>>4, chunk c&15.
    const uint64_t pol = evict_first_policy();
    auto issue = [&](uint32_t it) {
        if (it < nblk) {
            const uint32_t bb = b_first + it * bstep;
            const uint32_t sb = bb % cap;
            const uint32_t st = wbuf + (it % S) * kStage;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t c = lane + 32u * i;
                const uint32_t r = c >> 4, ch = c & 15u;
                const uint32_t slot = bb + r < row1 ? ring_slot(sb, r, cap) : sb;
                const uint64_t go = (uint64_t)slot * row_bytes + ch * 16u;
                const uint32_t so = r * 256u + ((ch ^ swz(r)) * 16u);
                cp_async16_ef(st + so, kbase + go, pol);
                cp_async16_ef(st + 4096u + so, vbase + go, pol);
            }
        }
        cp_async_commit();
    };

    // Optional q/k preparation (PREP = false compiles the plain kernel).  A
    // CTA that does not append starts its first loads before preparing, so
    // the preparation hides behind them; the appending CTA must store its
    // row before any load can read it.
    float *Qf = reinterpret_cast<float *>(smem_raw + NW * S * kStage + 2 * 8 * 32 * 16), *Kf = Qf + 16 * 128;
    const bool prep = PREP && J.qn != nullptr;
    const bool appender = J.k_new && row0 < row1 && row1 == J.end;
    // Under PDL the previous kernel on the stream may still be running until
    // griddepcontrol.wait returns, and only then are its writes visible.  The
    // host marks a job "pre" when that kernel cannot have written its cache
    // (see attention_jobs): such a CTA starts streaming its first rows before
    // the wait, overlapping the previous kernel's tail.  q, the gate and the
    // appended row may come from the previous kernel and are read after it.
    const bool pre_wait = J.pre != 0u && !appender;
    if (pre_wait) {
#pragma unroll
        for (int s = 0; s < S - 1; s++) issue(s);
    }
    griddep_wait();
    griddep_launch_dependents();
    // The gate factors of this CTA's heads, loaded now so the epilogue does
    // not wait on them (stored to shared memory after the q loads below).
    __shared__ float gate_s[16];
    const float gate_raw = (threadIdx.x < G && J.gate) ? J.gate[kvh * G + threadIdx.x] : 0.f;
    // A CTA that does not append starts its first loads before preparing q.
    const bool early = !pre_wait && !appender && prep;
    if (early) {
#pragma unroll
        for (int s = 0; s < S - 1; s++) issue(s);
    }
    if (prep) {
        prep_heads(P.rope[J.rope_idx], J, kvh, G, appender, Qf, Kf);
        __syncthreads();
    }
    if (warp < n_mt) {
        const uint32_t hg = warp * 8u + g;
        const bool valid = hg < G;
        const float *qp = prep ? Qf + (valid ? hg : 0u) * 128u : J.q + (uint64_t)(kvh * G + (valid ? hg : 0u)) * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            uint32_t r[4];
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const int w = 2 * kk + half;
                const uint32_t dim = (4u * (w >> 2) + t) * 8u + 2u * (w & 3);
                float2 x = valid ? *reinterpret_cast<const float2 *>(qp + dim) : make_float2(0.f, 0.f);
                x.x *= P.qscale;
                x.y *= P.qscale;
                const __half2 hi = __floats2half2_rn(x.x, x.y);
                const float2 hf = __half22float2(hi);
                const __half2 lo = __floats2half2_rn(x.x - hf.x, x.y - hf.y);
                r[half * 2] = h2_as_u32(hi);
                r[half * 2 + 1] = h2_as_u32(lo);
            }
            Qs[(warp * 8 + kk) * 32 + lane] = make_uint4(r[0], r[1], r[2], r[3]);
        }
    }
    if (threadIdx.x < G) gate_s[threadIdx.x] = J.gate ? sigmoid_dev(gate_raw) : 1.0f;
    fused_append<__half>(J, kvh, appender, P.kv_heads, prep ? Kf : nullptr);
    __syncthreads();

    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    if (!early && !pre_wait) {
#pragma unroll
        for (int s = 0; s < S - 1; s++) issue(s);
    }

    for (uint32_t it = 0; it < nblk; it++) {
        cp_async_wait<S - 2>();
        __syncwarp();
        issue(it + S - 1);
        const uint32_t b = b_first + it * bstep;
        const uint32_t st = wbuf + (it % S) * kStage;

        // S = q K^T for rows b .. b+15.
        float s[2][4];
#pragma unroll
        for (int i = 0; i < 2; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 a0 = lds128(qs_addr + (2 * c) * 512);
            const uint4 a1 = lds128(qs_addr + (2 * c + 1) * 512);
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const uint32_t r = 8u * i + g;
                const uint4 u = lds128(st + r * 256u + (((4u * c + t) ^ swz(r)) * 16u));
                mma16816(s[i], a0.x, a0.y, a0.z, a0.w, u.x, u.y);
                mma16816(s[i], a1.x, a1.y, a1.z, a1.w, u.z, u.w);
            }
        }

        float sc[2][2];
#pragma unroll
        for (int i = 0; i < 2; i++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const uint32_t r = b + 8u * i + 2u * t + e;
                sc[i][e] = r < row1 ? s[i][e] + s[i][e + 2] : -INFINITY;
            }
        float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        if (__any_sync(0xffffffffu, mx > m_run + kRescaleSlack)) {
            const float m_new = fmaxf(m_run, mx);
            const float alpha = fast_exp2(m_run - m_new);
            l_run *= alpha;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                o[i][0] *= alpha;
                o[i][1] *= alpha;
                o[i][2] *= alpha;
                o[i][3] *= alpha;
            }
            m_run = m_new;
        }
        uint32_t pa[4];
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const float p0 = fast_exp2(sc[i][0] - m_run), p1 = fast_exp2(sc[i][1] - m_run);
            l_run += p0 + p1;
            const __half2 hi = __floats2half2_rn(p0, p1);
            const float2 hf = __half22float2(hi);
            const __half2 lo = __floats2half2_rn(p0 - hf.x, p1 - hf.y);
            pa[2 * i] = h2_as_u32(hi);
            pa[2 * i + 1] = h2_as_u32(lo);
        }
        // V fragments: rows 2t, 2t+1, 2t+8, 2t+9; chunks g and g+8.
        uint4 vr[4][2];
#pragma unroll
        for (int x = 0; x < 4; x++) {
            const uint32_t r = 2u * t + (x & 1) + (x >> 1) * 8u;
            const uint32_t base = st + 4096u + r * 256u;
            vr[x][0] = lds128(base + ((g ^ swz(r)) * 16u));
            vr[x][1] = lds128(base + (((g + 8u) ^ swz(r)) * 16u));
        }
#pragma unroll
        for (int jt = 0; jt < 16; jt++) {
            const int u = jt >> 3, e = jt & 7, w = e >> 1;
            const uint32_t sel = (e & 1) ? 0x7632u : 0x5410u;
            const uint32_t b0 = prmt(word_of(vr[0][u], w), word_of(vr[1][u], w), sel);
            const uint32_t b1 = prmt(word_of(vr[2][u], w), word_of(vr[3][u], w), sel);
            mma16816(o[jt], pa[0], pa[1], pa[2], pa[3], b0, b1);
        }
        __syncwarp();
    }
    cp_async_wait<0>();
    __syncthreads();  // stage buffers become the epilogue arrays

    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    const uint32_t hrow = mt * 8u + g;
    const uint32_t orow = stream * 16u + hrow;
    if (hrow < G) {
#pragma unroll
        for (int jt = 0; jt < 16; jt++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const uint32_t c = 2u * t + e;
                const uint32_t dim = jt < 8 ? 8u * c + jt : 64u + 8u * c + (jt - 8);
                Os[os_at(orow, dim)] = o[jt][e] + o[jt][e + 2];
            }
        if (t == 0) {
            Ms[stream * 16u + hrow] = m_run;
            Ls[stream * 16u + hrow] = l_run;
        }
    }
    finish_cta<NW * 32>(P, J, j, kvh, split, cta, n_streams, Os, Ms, Ls, smem_raw, NW * S * kStage, gate_s);
}

// ------------------------------------------------------------ f32 kernel, tensor cores
// fp32 caches on the same per-warp cp.async pipeline and mma.sync tiles as
// the f16 kernel.  Every fp32 operand x is split into bf16 hi = rn(x) and
// lo = rn(x - hi) (16 significant bits, full fp32 range); S = q.K uses the
// M-row trick for q (rows 0-7 hi, 8-15 lo) against K_hi and then K_lo, and
// O = P.V likewise against V_hi and V_lo: four products, fp32 accumulate.
// Stage: K then V, 16 rows x 512 B each; 16-byte chunk ch of row r at slot
// ch ^ swz32(r), swz32(r) = ((r >> 1) & 3) ^ ((r & 1) << 2) (conflict free for
// both fragment patterns).  Dimension order inside a head: k-step kk, thread
// t holds dims 16kk + 4t .. +3 (one chunk); for PV, thread g holds dims
// 16g .. 16g+15 and n-tile jt is dim 16g + jt.
__device__ __forceinline__ uint32_t swz32(uint32_t r) { return ((r >> 1) & 3u) ^ ((r & 1u) << 2); }

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// (hi, lo) bf16 pairs of two floats: hi packs rn(a), rn(b); lo the residuals.
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

template <int NW, int S, bool PREP = false>
__global__ void __launch_bounds__(NW * 32, 1) decode_f32_pipe_kernel(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    constexpr uint32_t kStage = 16384;  // 16 rows x 512 B for K, then V
    uint4 *Qs = reinterpret_cast<uint4 *>(smem_raw + NW * S * kStage);  // [n_mt][8 kk][32 lanes]
    float *Os = reinterpret_cast<float *>(smem_raw);
    float *Ms = Os + NW * 16 * 128;
    float *Ls = Ms + 16 * NW;

    const uint32_t cta = blockIdx.x;
    const uint32_t j = locate_job(P, cta);
    const JobDev &J = P.job[j];
    const uint32_t local = cta - J.cta_begin;
    const uint32_t kvh = local / J.n_splits, split = local - kvh * J.n_splits;
    const uint32_t G = P.group;
    const uint32_t n_mt = (G + 7u) >> 3;
    const uint32_t n_streams = NW / n_mt;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t mt = warp % n_mt, stream = warp / n_mt;

    const uint32_t row0 = J.start + split * J.split_rows;
    const uint32_t row1 = min(row0 + J.split_rows, J.end);
    const uint32_t cap = J.cap;
    const uint64_t row_bytes = (uint64_t)P.kv_heads * 512u;
    const char *kbase = reinterpret_cast<const char *>(J.k) + kvh * 512u;
    const char *vbase = reinterpret_cast<const char *>(J.v) + kvh * 512u;
    const uint32_t qs_addr = (uint32_t)__cvta_generic_to_shared(Qs + mt * 8 * 32 + lane);
    const uint32_t wbuf = (uint32_t)__cvta_generic_to_shared(smem_raw) + warp * S * kStage;

    const uint32_t bstep = n_streams * 16u;
    const uint32_t b_first = row0 + stream * 16u;
    const uint32_t nblk = b_first < row1 ? (row1 - b_first + bstep - 1) / bstep : 0u;

    const uint64_t pol = evict_first_policy();
    auto issue = [&](uint32_t it) {
        if (it < nblk) {
            const uint32_t bb = b_first + it * bstep;
            const uint32_t sb = bb % cap;
            const uint32_t st = wbuf + (it % S) * kStage;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const uint32_t c = lane + 32u * i;
                const uint32_t r = c >> 5, ch = c & 31u;
                const uint32_t slot = bb + r < row1 ? ring_slot(sb, r, cap) : sb;
                const uint64_t go = (uint64_t)slot * row_bytes + ch * 16u;
                const uint32_t so = r * 512u + ((ch ^ swz32(r)) * 16u);
                cp_async16_ef(st + so, kbase + go, pol);
                cp_async16_ef(st + 8192u + so, vbase + go, pol);
            }
        }
        cp_async_commit();
    };

    // Optional q/k preparation (PREP = false compiles the plain kernel).  A
    // CTA that does not append starts its first loads before preparing, so
    // the preparation hides behind them; the appending CTA must store its
    // row before any load can read it.
    float *Qf = reinterpret_cast<float *>(smem_raw + NW * S * kStage + 2 * 8 * 32 * 16), *Kf = Qf + 16 * 128;
    const bool prep = PREP && J.qn != nullptr;
    const bool appender = J.k_new && row0 < row1 && row1 == J.end;
    // Under PDL the previous kernel on the stream may still be running until
    // griddepcontrol.wait returns, and only then are its writes visible.  The
    // host marks a job "pre" when that kernel cannot have written its cache
    // (see attention_jobs): such a CTA starts streaming its first rows before
    // the wait, overlapping the previous kernel's tail.  q, the gate and the
    // appended row may come from the previous kernel and are read after it.
    const bool pre_wait = J.pre != 0u && !appender;
    if (pre_wait) {
#pragma unroll
        for (int s = 0; s < S - 1; s++) issue(s);
    }
    griddep_wait();
    griddep_launch_dependents();
    // The gate factors of this CTA's heads, loaded now so the epilogue does
    // not wait on them (stored to shared memory after the q loads below).
    __shared__ float gate_s[16];
    const float gate_raw = (threadIdx.x < G && J.gate) ? J.gate[kvh * G + threadIdx.x] : 0.f;
    // A CTA that does not append starts its first loads before preparing q.
    const bool early = !pre_wait && !appender && prep;
    if (early) {
#pragma unroll
        for (int s = 0; s < S - 1; s++) issue(s);
    }
    if (prep) {
        prep_heads(P.rope[J.rope_idx], J, kvh, G, appender, Qf, Kf);
        __syncthreads();
    }
    if (warp < n_mt) {
        const uint32_t hg = warp * 8u + g;
        const bool valid = hg < G;
        const float *qp = prep ? Qf + (valid ? hg : 0u) * 128u : J.q + (uint64_t)(kvh * G + (valid ? hg : 0u)) * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            const float4 x = valid ? *reinterpret_cast<const float4 *>(qp + 16 * kk + 4 * t)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            uint32_t r0, r1, r2, r3;
            split2(x.x * P.qscale, x.y * P.qscale, r0, r1);
            split2(x.z * P.qscale, x.w * P.qscale, r2, r3);
            Qs[(warp * 8 + kk) * 32 + lane] = make_uint4(r0, r1, r2, r3);
        }
    }
    if (threadIdx.x < G) gate_s[threadIdx.x] = J.gate ? sigmoid_dev(gate_raw) : 1.0f;
    fused_append<float>(J, kvh, appender, P.kv_heads, prep ? Kf : nullptr);
    __syncthreads();

    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    if (!early && !pre_wait) {
#pragma unroll
        for (int s = 0; s < S - 1; s++) issue(s);
    }

    for (uint32_t it = 0; it < nblk; it++) {
        cp_async_wait<S - 2>();
        __syncwarp();
        issue(it + S - 1);
        const uint32_t b = b_first + it * bstep;
        const uint32_t st = wbuf + (it % S) * kStage;

        float s[2][4];
#pragma unroll
        for (int i = 0; i < 2; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            const uint4 a = lds128(qs_addr + kk * 512);
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const uint32_t r = 8u * i + g;
                const uint4 u = lds128(st + r * 512u + (((4u * kk + t) ^ swz32(r)) * 16u));
                uint32_t h0, l0, h1, l1;
                split2(__uint_as_float(u.x), __uint_as_float(u.y), h0, l0);
                split2(__uint_as_float(u.z), __uint_as_float(u.w), h1, l1);
                mma_bf16(s[i], a.x, a.y, a.z, a.w, h0, h1);
                mma_bf16(s[i], a.x, a.y, a.z, a.w, l0, l1);
            }
        }

        float sc[2][2];
#pragma unroll
        for (int i = 0; i < 2; i++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const uint32_t r = b + 8u * i + 2u * t + e;
                sc[i][e] = r < row1 ? s[i][e] + s[i][e + 2] : -INFINITY;
            }
        float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        if (__any_sync(0xffffffffu, mx > m_run + kRescaleSlack)) {
            const float m_new = fmaxf(m_run, mx);
            const float alpha = fast_exp2(m_run - m_new);
            l_run *= alpha;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                o[i][0] *= alpha;
                o[i][1] *= alpha;
                o[i][2] *= alpha;
                o[i][3] *= alpha;
            }
            m_run = m_new;
        }
        uint32_t pa[4];
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const float p0 = fast_exp2(sc[i][0] - m_run), p1 = fast_exp2(sc[i][1] - m_run);
            l_run += p0 + p1;
            split2(p0, p1, pa[2 * i], pa[2 * i + 1]);
        }
        // V: rows 2t, 2t+1, 2t+8, 2t+9; dims 16g .. 16g+15 (chunks 4g .. 4g+3).
#pragma unroll
        for (int c4 = 0; c4 < 4; c4++) {
            float4 vv[4];
#pragma unroll
            for (int x = 0; x < 4; x++) {
                const uint32_t r = 2u * t + (x & 1) + (x >> 1) * 8u;
                const uint4 u = lds128(st + 8192u + r * 512u + (((4u * g + c4) ^ swz32(r)) * 16u));
                vv[x] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                                    __uint_as_float(u.w));
            }
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int jt = c4 * 4 + e;
                const float a0 = e == 0 ? vv[0].x : e == 1 ? vv[0].y : e == 2 ? vv[0].z : vv[0].w;
                const float a1 = e == 0 ? vv[1].x : e == 1 ? vv[1].y : e == 2 ? vv[1].z : vv[1].w;
                const float a2 = e == 0 ? vv[2].x : e == 1 ? vv[2].y : e == 2 ? vv[2].z : vv[2].w;
                const float a3 = e == 0 ? vv[3].x : e == 1 ? vv[3].y : e == 2 ? vv[3].z : vv[3].w;
                uint32_t h0, l0, h1, l1;
                split2(a0, a1, h0, l0);
                split2(a2, a3, h1, l1);
                mma_bf16(o[jt], pa[0], pa[1], pa[2], pa[3], h0, h1);
                mma_bf16(o[jt], pa[0], pa[1], pa[2], pa[3], l0, l1);
            }
        }
        __syncwarp();
    }
    cp_async_wait<0>();
    __syncthreads();

    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    const uint32_t hrow = mt * 8u + g;
    const uint32_t orow = stream * 16u + hrow;
    if (hrow < G) {
#pragma unroll
        for (int jt = 0; jt < 16; jt++)
#pragma unroll
            for (int e = 0; e < 2; e++) Os[os_at(orow, 16u * (2u * t + e) + jt)] = o[jt][e] + o[jt][e + 2];
        if (t == 0) {
            Ms[stream * 16u + hrow] = m_run;
            Ls[stream * 16u + hrow] = l_run;
        }
    }
    finish_cta<NW * 32>(P, J, j, kvh, split, cta, n_streams, Os, Ms, Ls, smem_raw, NW * S * kStage, gate_s);
}

// ------------------------------------------------------------ generic kernel
// Any head_dim <= 256 and any group: one warp per (job, query head), one
// pass over the rows with an online softmax.  Lane holds dims lane + 32*i.
struct GenericParams {
    JobDev job[kMaxJobs];
    uint32_t n_jobs, q_heads, kv_heads, head_dim;
    float scale;
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T>
__global__ void __launch_bounds__(256) decode_generic_kernel(const __grid_constant__ GenericParams P) {
    const uint32_t gw = blockIdx.x * 8u + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t jj = gw / P.q_heads;
    if (jj >= P.n_jobs) return;
    const uint32_t h = gw - jj * P.q_heads;
    const JobDev &J = P.job[jj];
    const uint32_t G = P.q_heads / P.kv_heads;
    const uint32_t kvh = h / G;
    const uint32_t hd = P.head_dim;
    const uint64_t row = (uint64_t)P.kv_heads * hd;
    const T *kc = reinterpret_cast<const T *>(J.k) + (uint64_t)kvh * hd;
    const T *vc = reinterpret_cast<const T *>(J.v) + (uint64_t)kvh * hd;
    float q[8], o[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t d = lane + 32u * i;
        q[i] = d < hd ? J.q[(uint64_t)h * hd + d] * P.scale : 0.f;
        o[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (uint32_t r = J.start; r < J.end; r++) {
        const uint64_t slot = r % J.cap;
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t d = lane + 32u * i;
            if (d < hd) dot += q[i] * to_f<T>(kc[slot * row + d]);
        }
        for (int msk = 16; msk; msk >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, msk);
        const float mn = fmaxf(m, dot);
        const float alpha = exp2f(m - mn), p = exp2f(dot - mn);
        l = l * alpha + p;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t d = lane + 32u * i;
            o[i] = o[i] * alpha + (d < hd ? p * to_f<T>(vc[slot * row + d]) : 0.f);
        }
        m = mn;
    }
    const float g = J.gate ? sigmoid_dev(J.gate[h]) : 1.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t d = lane + 32u * i;
        if (d < hd) J.out[(uint64_t)h * hd + d] = l > 0.f ? o[i] / l * g : 0.f;
    }
}

// ------------------------------------------------------------ host side
// inv_freq of RoPE pair `pair`: sf37_inv_freq (sf37.c:1995-2013), double.
static double rope_inv_freq(uint32_t pair, uint32_t dim, double theta, uint32_t llama3) {
    const double inv = 1.0 / pow(theta, (double)(pair * 2u) / (double)dim);
    if (!llama3) return inv;
    const double factor = 2.0, low_ff = 1.0, high_ff = 32.0, old_ctx = 131072.0;
    const double low_wl = old_ctx / low_ff, high_wl = old_ctx / high_ff;
    const double wavelen = 2.0 * 3.14159265358979323846 / inv;
    if (wavelen > low_wl) return inv / factor;
    if (wavelen < high_wl) return inv;
    const double smooth = (old_ctx / wavelen - low_ff) / (high_ff - low_ff);
    return (1.0 - smooth) * inv / factor + smooth * inv;
}

// cos/sin of pair i at position pos, exactly as apply_rope_one computes
// them on the CPU (sf37.c:2020-2024): libm cosf / sinf of the float angle.
struct RopeKey {
    uint32_t rotary, llama3, pos;
    double theta;
    bool operator==(const RopeKey &o) const {
        return rotary == o.rotary && llama3 == o.llama3 && pos == o.pos && theta == o.theta;
    }
};

static void rope_table(float *t, const RopeKey &k) {
    for (uint32_t i = 0; i < 64; i++) {
        t[i] = 1.f;
        t[64 + i] = 0.f;
        if (i < k.rotary / 2u) {
            const float ang = (float)((double)k.pos * rope_inv_freq(i, k.rotary, k.theta, k.llama3));
            t[i] = cosf(ang);
            t[64 + i] = sinf(ang);
        }
    }
}

constexpr size_t kPrepSmem = (16 * 128 + 128) * 4;  // prepared q heads + K head (PREP kernels)
static size_t smem_pipe(int nw, int stages) { return (size_t)nw * stages * 8192 + 2 * 8 * 32 * 16; }
static size_t smem_pipe32(int nw, int stages) { return (size_t)nw * stages * 16384 + 2 * 8 * 32 * 16; }
static int launch_generic(const AttnJob *jobs, uint32_t n, uint32_t q_heads, uint32_t kv_heads,
                          uint32_t head_dim, int dtype, cudaStream_t stream) {
    if (head_dim > 256)
        return set_error(SF37KV_EUNSUPPORTED, "attention: head_dim %u > 256", head_dim);
    for (uint32_t base = 0; base < n; base += kMaxJobs) {
        GenericParams P;
        P.n_jobs = 0;
        P.q_heads = q_heads;
        P.kv_heads = kv_heads;
        P.head_dim = head_dim;
        P.scale = kLog2e / sqrtf((float)head_dim);
        for (uint32_t i = base; i < n && i < base + kMaxJobs; i++) {
            const AttnJob &A = jobs[i];
            JobDev &D = P.job[P.n_jobs++];
            D = JobDev{A.k, A.v, A.q, A.gate, A.out, A.start, A.end, A.cap, 0, 1, 0, nullptr, nullptr, 0};
        }
        const uint64_t warps = (uint64_t)P.n_jobs * q_heads;
        const unsigned grid = (unsigned)((warps + 7) / 8);
        if (dtype == SF37KV_F32) decode_generic_kernel<float><<<grid, 256, 0, stream>>>(P);
        else decode_generic_kernel<__half><<<grid, 256, 0, stream>>>(P);
        g_launches++;
        if (int rc = check_cuda(cudaGetLastError(), "generic attention launch")) return rc;
    }
    return SF37KV_OK;
}

// Batched f16 kernel: 4 warps, two CTAs per SM.  Small-launch f16 kernel:
// 8 warps, one CTA per SM (its stage buffers hold every split partial of a
// group for the merge).  f32 kernel: 4 warps, one CTA per SM.
static const size_t kSmemF16 = smem_pipe(4, 3), kSmemF16Wide = smem_pipe(8, 3), kSmemF32 = smem_pipe32(4, 3);

// What the last decode kernel launched on each stream appended to.  The
// decode kernels trigger their dependents early (PDL), so the next decode on
// the same stream may start while one is still running; a job of the new
// launch may stream its rows before griddepcontrol.wait only if the running
// kernel cannot write them, i.e. it appended to neither of the job's caches
// (sf37kv_decode_noalloc's kernel records its appends here too).  Kernels
// that this file does not launch (other libraries', this library's appends
// and prefills) trigger no early start, so a decode that follows one of them
// starts after it has completed whatever the record says; with no record for
// a stream, no job streams early.
struct StreamRecord {
    cudaStream_t stream;
    bool used;
    uint32_t n;
    const void *caches[2 * kMaxJobs];
};
static StreamRecord g_stream_rec[8];
static uint32_t g_stream_rec_next = 0;
static std::mutex g_stream_rec_mu;

// Marks each job of a launch on `s` that may stream before the wait.
static void mark_pre(cudaStream_t s, JobDev *jobs, uint32_t n) {
    std::lock_guard<std::mutex> lk(g_stream_rec_mu);
    const StreamRecord *r = nullptr;
    for (const StreamRecord &x : g_stream_rec)
        if (x.used && x.stream == s) r = &x;
    for (uint32_t i = 0; i < n; i++) {
        bool ok = r != nullptr;
        for (uint32_t c = 0; ok && r && c < r->n; c++) ok = r->caches[c] != jobs[i].k && r->caches[c] != jobs[i].v;
        jobs[i].pre = ok ? 1u : 0u;
    }
}

void note_stream_appends(cudaStream_t s, const JobDev *jobs, uint32_t n) {
    std::lock_guard<std::mutex> lk(g_stream_rec_mu);
    StreamRecord *r = nullptr;
    for (StreamRecord &x : g_stream_rec)
        if (x.used && x.stream == s) r = &x;
    if (!r) {
        r = &g_stream_rec[g_stream_rec_next];
        g_stream_rec_next = (g_stream_rec_next + 1u) % 8u;
    }
    r->stream = s;
    r->used = true;
    r->n = 0;
    for (uint32_t i = 0; i < n && r->n + 2u <= 2u * kMaxJobs; i++) {
        if (!jobs[i].k_new) continue;
        r->caches[r->n++] = jobs[i].k;
        r->caches[r->n++] = jobs[i].v;
    }
}

// Launches a pipelined decode kernel of `warps` warps; with P.pdl, with
// programmatic stream serialization (its CTAs start while the previous kernel
// on the stream drains and wait in griddepcontrol.wait).
template <typename Kernel>
static void launch_decode(Kernel kernel, unsigned grid, unsigned warps, size_t smem, cudaStream_t s,
                          const DecodeParams &P) {
    // Kernel attributes, once per kernel instance (the instances share one
    // function-pointer type, so they are told apart by address).
    static const void *done[16];
    static int n_done = 0;
    bool seen = false;
    for (int i = 0; i < n_done; i++) seen |= done[i] == (const void *)kernel;
    if (!seen) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (n_done < 16) done[n_done++] = (const void *)kernel;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(warps * 32u);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = P.pdl ? 1 : 0;
    (void)cudaLaunchKernelEx(&cfg, kernel, P);
}

int attention_jobs(const AttnJob *jobs, uint32_t n, uint32_t q_heads, uint32_t kv_heads,
                   uint32_t head_dim, int dtype, cudaStream_t stream) {
    if (dtype != SF37KV_F32 && dtype != SF37KV_F16)
        return set_error(SF37KV_EINVAL, "attention: unknown cache dtype %d", dtype);
    if (kv_heads == 0 || q_heads == 0 || q_heads % kv_heads != 0 || head_dim == 0)
        return set_error(SF37KV_EINVAL, "attention: bad head configuration q=%u kv=%u d=%u",
                         q_heads, kv_heads, head_dim);
    for (uint32_t i = 0; i < n; i++) {
        const AttnJob &A = jobs[i];
        if (!A.k || !A.v || !A.q || !A.out || A.cap == 0 || A.end < A.start)
            return set_error(SF37KV_EINVAL, "attention: job %u is invalid", i);
    }
    const uint32_t G = q_heads / kv_heads;
    // The pipelined kernels (head_dim 128, group <= 16) store the appended
    // rows themselves; for the generic kernel they are appended by a
    // separate launch first.
    const bool fuses = head_dim == 128 && G <= 16;
    bool any_prep = false;
    for (uint32_t i = 0; i < n; i++) any_prep |= jobs[i].prep != nullptr;
    if (any_prep && !fuses)
        return set_error(SF37KV_EUNSUPPORTED,
                         "decode_prep: needs head_dim 128 and group <= 16");
    if (!fuses) {
        AppendJob aj[kMaxJobs];
        for (uint32_t base = 0; base < n; base += kMaxJobs) {
            uint32_t na = 0;
            for (uint32_t i = base; i < n && i < base + kMaxJobs; i++)
                if (jobs[i].k_new)
                    aj[na++] = AppendJob{const_cast<void *>(jobs[i].k), const_cast<void *>(jobs[i].v), jobs[i].k_new,
                                         jobs[i].v_new, jobs[i].end - 1u, 1, jobs[i].cap};
            if (na)
                if (int rc = append_jobs(aj, na, kv_heads * head_dim, dtype, stream)) return rc;
        }
    }
    if (!fuses) return launch_generic(jobs, n, q_heads, kv_heads, head_dim, dtype, stream);

    const int sms = num_sms();
    for (uint32_t base = 0, m = 0; base < n; base += m) {
        m = (n - base) < (uint32_t)kMaxJobs ? (n - base) : (uint32_t)kMaxJobs;
        // q/k preparation: at most kMaxRope distinct RoPE tables per launch
        RopeKey keys[kMaxRope];
        uint32_t n_keys = 0, rope_idx[kMaxJobs] = {};
        for (uint32_t i = 0; i < m; i++) {
            const AttnJob &A = jobs[base + i];
            if (!A.prep) continue;
            const RopeKey k{A.prep->rotary_dim, A.prep->llama3, A.end - 1u, A.prep->theta};
            uint32_t f = 0;
            while (f < n_keys && !(keys[f] == k)) f++;
            if (f == n_keys) {
                if (n_keys == (uint32_t)kMaxRope) {
                    m = i;  // the rest goes to the next launch
                    break;
                }
                keys[n_keys++] = k;
            }
            rope_idx[i] = f;
        }
        uint64_t total = 0;
        for (uint32_t i = 0; i < m; i++) total += (uint64_t)(jobs[base + i].end - jobs[base + i].start);
        total *= kv_heads;
        // Rows per CTA.  Big batches (e.g. 48 layers x 32K rows): about 8
        // waves of resident CTAs, which keeps the last partial wave small.
        // Small launches (one layer): a single wave, so each (layer, KV head)
        // has few splits and its last CTA merges few partials.
        const uint64_t occ = dtype == SF37KV_F16 ? 2 : 1;  // resident CTAs per SM
        uint64_t per = (total + (uint64_t)sms * 24 - 1) / ((uint64_t)sms * 24);
        if (per < 2048) {
            const uint64_t slots = (uint64_t)sms * occ;
            per = (total + slots - 1) / slots;
            // round so that ceil(rows / per) CTAs of a job stay within the wave
            per = ((per + 127) / 128) * 128;
            if (per < 128) per = 128;
            const uint64_t ctas1 = (uint64_t)m * kv_heads;
            uint64_t longest = 0;
            for (uint32_t i = 0; i < m; i++) longest = std::max<uint64_t>(longest, jobs[base + i].end - jobs[base + i].start);
            // Jobs of very different lengths (full and sliding layers): size
            // CTAs by rows, not by jobs, so one long job's splits do not pile
            // onto a few SMs (config 3 on 2 GPUs: 192 groups, 48 of them 65K
            // rows, the rest 512).
            const bool mixed = longest * ctas1 > 2u * total;
            if (ctas1 <= slots && !mixed) {
                // Per-job split count (jobs of similar length): the one whose
                // CTAs fill whole waves best, i.e. the fewest waves per unit of
                // work, ceil(ns * ctas1 / slots) / ns; ties go to fewer splits
                // (cheaper merge).  E.g. 192 groups on 296 slots: 3 splits
                // (1.95 waves) rather than 1 (192 CTAs, 44 SMs doubly loaded).
                uint64_t ns = 1;
                double best = 1e30;
                for (uint64_t c = 1; c <= slots / ctas1 * 2 + 2 && c <= kMaxSplits; c++) {
                    const double cost = (double)((c * ctas1 + slots - 1) / slots) / (double)c;
                    if (cost < best * 0.95) {
                        best = cost;
                        ns = c;
                    }
                }
                per = ((longest + ns - 1) / ns + 127) / 128 * 128;
                if (per < 128) per = 128;
            } else if (per > 8192 || mixed) {
                // More (layer, head) groups than one wave holds, with a few
                // long jobs among many short ones (config 3: 12 full layers of
                // 65K rows and 36 sliding layers of 512): one-wave sizing makes
                // the long jobs' CTAs huge, and their tail cannot overlap the
                // next launch.  Measured on config 3: 21.6K rows per CTA 1682
                // tok/s, 8192 rows 2002 tok/s.
                if (per > 8192) per = 8192;
            }
        }
        DecodeParams P;
        P.pdl = 0;
        P.n_jobs = m;
        P.q_heads = q_heads;
        P.kv_heads = kv_heads;
        P.group = G;
        P.part_stride = (G * 130u + 3u) & ~3u;
        P.qscale = kLog2e / sqrtf(128.0f);
        for (uint32_t f = 0; f < n_keys; f++) rope_table(P.rope[f], keys[f]);
        P.gat = g_gather_cur ? *g_gather_cur : GatherDev{};
        // Small launches (a single layer or a few: at most one (job, KV
        // head) group per two SMs) run one CTA per SM: the f16 kernel in its
        // 8-warp form, and ns = SMs / groups splits per group, so the split
        // partials of a group fit the merging CTA's stage buffers in one
        // pass.  Larger launches keep the plan above.
        const uint32_t groups = m * kv_heads;
        const bool small = groups * 2u <= (uint32_t)sms;
        const int slot = (dtype == SF37KV_F16 ? 0 : 2) + (any_prep ? 1 : 0);
        P.err = device_error_flag();
        uint32_t ctas = 0;
        bool any_split = false;
        for (uint32_t i = 0; i < m; i++) {
            const AttnJob &A = jobs[base + i];
            const uint32_t rows = A.end - A.start;
            uint64_t ns;
            uint32_t sr;
            if (small) {
                // splits in proportion to the job's share of all rows
                ns = (uint64_t)sms * rows / (total ? total : 1);
                if (ns < 1) ns = 1;
                if (ns > kMaxSplits) ns = kMaxSplits;
                sr = (uint32_t)((rows + ns - 1) / ns);
                sr = (sr + 15u) & ~15u;
                if (sr == 0) sr = 16;
            } else {
                ns = (rows + per - 1) / per;
                if (ns < 1) ns = 1;
                if (ns > kMaxSplits) ns = kMaxSplits;
                sr = (uint32_t)((rows + ns - 1) / ns);
                sr = (sr + 127u) & ~127u;
                if (sr == 0) sr = 128;
            }
            ns = (rows + sr - 1) / sr;
            if (ns < 1) ns = 1;
            if (ns > 1) any_split = true;
            JobDev &D = P.job[i];
            D = JobDev{A.k, A.v, A.q, A.gate, A.out, A.start, A.end, A.cap, sr, (uint32_t)ns, ctas,
                       fuses ? A.k_new : nullptr, fuses ? A.v_new : nullptr,
                       g_gather_cur ? g_gather_off[base + i] : 0};
            if (A.prep) {
                D.qn = A.prep->q_norm;
                D.kn = A.prep->k_norm;
                D.rotary = A.prep->rotary_dim;
                D.rope_idx = rope_idx[i];
                D.eps = A.prep->eps;
            }
            if ((uint64_t)ctas + ns * kv_heads > 0x7fffffffull)
                return set_error(SF37KV_EINVAL, "attention: grid too large");
            ctas += (uint32_t)ns * kv_heads;
        }
        P.total_ctas = ctas;
        if (P.gat.world) P.gat.total_groups = groups;
        Scratch S;
        if (any_split) {
            if (int rc = scratch_get((uint64_t)ctas * P.part_stride * 4u, (uint64_t)m * kv_heads, &S))
                return rc;
        }
        P.part = S.part;
        P.counters = S.counters;
        // Pipelined kernels, launched with programmatic dependent launch (PDL).
        P.pdl = 1;
        mark_pre(stream, P.job, m);
        note_stream_appends(stream, P.job, m);
        switch (slot * 2 + (small ? 1 : 0)) {
            case 0: launch_decode(decode_f16_pipe_kernel<4, 3, false>, ctas, 4, kSmemF16, stream, P); break;
            case 1: launch_decode(decode_f16_pipe_kernel<8, 3, false>, ctas, 8, kSmemF16Wide, stream, P); break;
            case 2: launch_decode(decode_f16_pipe_kernel<4, 3, true>, ctas, 4, kSmemF16 + kPrepSmem, stream, P); break;
            case 3: launch_decode(decode_f16_pipe_kernel<8, 3, true>, ctas, 8, kSmemF16Wide + kPrepSmem, stream, P); break;
            case 4:
            case 5: launch_decode(decode_f32_pipe_kernel<4, 3, false>, ctas, 4, kSmemF32, stream, P); break;
            default: launch_decode(decode_f32_pipe_kernel<4, 3, true>, ctas, 4, kSmemF32 + kPrepSmem, stream, P); break;
        }
        g_launches++;
        if (int rc = check_cuda(cudaGetLastError(), "attention launch")) return rc;
    }
    return SF37KV_OK;
}

}  // namespace sf37kv

using namespace sf37kv;

// ------------------------------------------------------------ native API
static int decode_layers(const sf37kv_decode_layer *layers, const sf37kv_qk_prep *prep, uint32_t n_layers,
                         uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, int dtype, void *stream) {
    if (!layers && n_layers) return set_error(SF37KV_EINVAL, "decode: layers is NULL");
    cudaStream_t s = stream ? (cudaStream_t)stream : current_stream();
    AttnJob jobs[kMaxJobs];
    for (uint32_t base = 0; base < n_layers; base += kMaxJobs) {
        uint32_t m = 0;
        for (uint32_t i = base; i < n_layers && m < (uint32_t)kMaxJobs; i++, m++) {
            const sf37kv_decode_layer &L = layers[i];
            if (L.cache.cap == 0) return set_error(SF37KV_EINVAL, "decode: layer %u cap 0", i);
            if ((L.k_new != nullptr) != (L.v_new != nullptr))
                return set_error(SF37KV_EINVAL, "decode: layer %u has only one of k_new/v_new", i);
            if (L.k_new && (((uintptr_t)L.k_new | (uintptr_t)L.v_new) & 15u))
                return set_error(SF37KV_EINVAL, "decode: layer %u k_new/v_new must be 16-byte aligned", i);
            jobs[m] = AttnJob{L.cache.k_cache, L.cache.v_cache, L.q, L.gate, L.out,
                              start_at(L.pos, L.cache.cap, L.cache.sliding, L.cache.window),
                              L.pos + 1u, L.cache.cap, L.k_new, L.v_new, prep ? &prep[i] : nullptr};
            if (prep) {
                const sf37kv_qk_prep &Q = prep[i];
                if (!Q.q_norm || (L.k_new && !Q.k_norm))
                    return set_error(SF37KV_EINVAL, "decode_prep: layer %u norm weight is NULL", i);
                if (Q.rotary_dim == 0 || Q.rotary_dim > head_dim || (Q.rotary_dim & 1u))
                    return set_error(SF37KV_EINVAL, "decode_prep: layer %u rotary_dim %u must be even and <= %u",
                                     i, Q.rotary_dim, head_dim);
                if ((((uintptr_t)L.q | (uintptr_t)Q.q_norm | (uintptr_t)Q.k_norm) & 7u) ||
                    ((uintptr_t)L.q & 15u))
                    return set_error(SF37KV_EINVAL, "decode_prep: layer %u q must be 16-byte and the weights "
                                                    "8-byte aligned", i);
            }
        }
        if (int rc = attention_jobs(jobs, m, q_heads, kv_heads, head_dim, dtype, s)) return rc;
    }
    return SF37KV_OK;
}

extern "C" int sf37kv_decode(const sf37kv_decode_layer *layers, uint32_t n_layers, uint32_t q_heads,
                             uint32_t kv_heads, uint32_t head_dim, int dtype, void *stream) {
    return decode_layers(layers, nullptr, n_layers, q_heads, kv_heads, head_dim, dtype, stream);
}

extern "C" int sf37kv_decode_prep(const sf37kv_decode_layer *layers, const sf37kv_qk_prep *prep,
                                  uint32_t n_layers, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                                  int dtype, void *stream) {
    if (!prep && n_layers) return set_error(SF37KV_EINVAL, "decode_prep: prep is NULL");
    if (head_dim != 128) return set_error(SF37KV_EUNSUPPORTED, "decode_prep: head_dim must be 128");
    return decode_layers(layers, prep, n_layers, q_heads, kv_heads, head_dim, dtype, stream);
}

// ------------------------------------------------------------ drop-in API
static int dropin_fail(const char *what) {
    fprintf(stderr, "sf37: %s failed: %s\n", what, sf37kv_last_error());
    return 0;
}

extern "C" int sf37_cuda_attention_decode_heads(sf37_cuda_tensor *out_heads, const sf37_cuda_tensor *q,
                                                const sf37_cuda_tensor *k_cache,
                                                const sf37_cuda_tensor *v_cache,
                                                const sf37_cuda_tensor *head_gate, uint32_t n_cache,
                                                uint32_t cache_cap, uint32_t q_heads,
                                                uint32_t kv_heads, uint32_t head_dim, int sliding,
                                                uint32_t window) {
    // Validation as sf37_cuda.cu:3015-3024.
    if (!out_heads || !q || !k_cache || !v_cache || !head_gate || kv_heads == 0 ||
        q_heads % kv_heads != 0 || n_cache > cache_cap)
        return 0;
    const uint64_t q_dim = (uint64_t)q_heads * head_dim, kv_dim = (uint64_t)kv_heads * head_dim;
    if (out_heads->bytes < q_dim * 4 || q->bytes < q_dim * 4 ||
        k_cache->bytes < (uint64_t)cache_cap * kv_dim * 4 ||
        v_cache->bytes < (uint64_t)cache_cap * kv_dim * 4 || head_gate->bytes < (uint64_t)q_heads * 4)
        return 0;
    uint32_t start = 0;
    if (sliding && n_cache > window) start = n_cache - window;
    AttnJob job{k_cache->ptr, v_cache->ptr, (const float *)q->ptr, (const float *)head_gate->ptr,
                (float *)out_heads->ptr, start, n_cache, cache_cap};
    if (attention_jobs(&job, 1, q_heads, kv_heads, head_dim, SF37KV_F32, current_stream()))
        return dropin_fail("attention_decode_heads");
    return 1;
}

extern "C" int sf37_cuda_attention_decode_heads_at(sf37_cuda_tensor *out_heads, const sf37_cuda_tensor *q,
                                                   const sf37_cuda_tensor *k_cache,
                                                   const sf37_cuda_tensor *v_cache,
                                                   const sf37_cuda_tensor *head_gate, uint32_t pos,
                                                   uint32_t cache_cap, uint32_t q_heads,
                                                   uint32_t kv_heads, uint32_t head_dim, int sliding,
                                                   uint32_t window) {
    // Validation as sf37_cuda.cu:3091-3103.
    if (!out_heads || !q || !k_cache || !v_cache || !head_gate || cache_cap == 0 ||
        kv_heads == 0 || q_heads % kv_heads != 0 || head_dim == 0)
        return 0;
    const uint64_t q_dim = (uint64_t)q_heads * head_dim, kv_dim = (uint64_t)kv_heads * head_dim;
    if (out_heads->bytes < q_dim * 4 || q->bytes < q_dim * 4 ||
        k_cache->bytes < (uint64_t)cache_cap * kv_dim * 4 ||
        v_cache->bytes < (uint64_t)cache_cap * kv_dim * 4 || head_gate->bytes < (uint64_t)q_heads * 4)
        return 0;
    AttnJob job{k_cache->ptr, v_cache->ptr, (const float *)q->ptr, (const float *)head_gate->ptr,
                (float *)out_heads->ptr, start_at(pos, cache_cap, sliding, window), pos + 1u, cache_cap};
    if (attention_jobs(&job, 1, q_heads, kv_heads, head_dim, SF37KV_F32, current_stream()))
        return dropin_fail("attention_decode_heads_at");
    return 1;
}

__global__ static void gqa_single_token_kernel(float *out, const float *v, const float *gate,
                                               uint32_t q_heads, uint32_t kv_heads, uint32_t hd) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)q_heads * hd) return;
    const uint32_t h = (uint32_t)(i / hd), d = (uint32_t)(i - (uint64_t)h * hd);
    const uint32_t kvh = h / (q_heads / kv_heads);
    out[i] = v[(uint64_t)kvh * hd + d] * sigmoid_dev(gate[h]);
}

// sf37_cuda.cu:2333-2367.
extern "C" int sf37_cuda_gqa_single_token_heads(sf37_cuda_tensor *out_heads, const sf37_cuda_tensor *v,
                                                const sf37_cuda_tensor *head_gate, uint32_t q_heads,
                                                uint32_t kv_heads, uint32_t head_dim) {
    if (!out_heads || !v || !head_gate || kv_heads == 0 || q_heads % kv_heads != 0) return 0;
    const uint64_t q_dim = (uint64_t)q_heads * head_dim, kv_dim = (uint64_t)kv_heads * head_dim;
    if (out_heads->bytes < q_dim * 4 || v->bytes < kv_dim * 4 || head_gate->bytes < (uint64_t)q_heads * 4)
        return 0;
    if (q_dim == 0) return 1;
    gqa_single_token_kernel<<<(unsigned)((q_dim + 255) / 256), 256, 0, current_stream()>>>(
        (float *)out_heads->ptr, (const float *)v->ptr, (const float *)head_gate->ptr, q_heads,
        kv_heads, head_dim);
    g_launches++;
    if (check_cuda(cudaGetLastError(), "gqa single-token launch")) return dropin_fail("gqa_single_token_heads");
    return 1;
}

// ------------------------------------------------------------ caller-provided scratch
// Split-K decode launch whose partials and counters live in memory the
// caller provides (the allocation-free entry point, decode_noalloc.cu).  It
// plans like attention_jobs but raises the rows per CTA until the partials
// fit in part_bytes, and never allocates.  Only the fast kernels (head_dim
// 128, group <= 16) are reachable here; other shapes are rejected.
namespace sf37kv {

int attention_jobs_prealloc(const AttnJob *jobs, uint32_t n, uint32_t q_heads, uint32_t kv_heads,
                            uint32_t head_dim, int dtype, cudaStream_t stream, float *part,
                            uint64_t part_bytes, uint32_t *counters, uint64_t n_counters) {
    if (dtype != SF37KV_F32 && dtype != SF37KV_F16)
        return set_error(SF37KV_EINVAL, "decode_noalloc: unknown cache dtype %d", dtype);
    if (kv_heads == 0 || q_heads == 0 || q_heads % kv_heads != 0)
        return set_error(SF37KV_EINVAL, "decode_noalloc: bad head configuration q=%u kv=%u", q_heads,
                         kv_heads);
    const uint32_t G = q_heads / kv_heads;
    if (head_dim != 128 || G > 16)
        return set_error(SF37KV_EUNSUPPORTED,
                         "decode_noalloc: needs head_dim 128 and q_heads/kv_heads <= 16; got head_dim %u, group %u",
                         head_dim, G);
    if (n > (uint32_t)kMaxJobs)
        return set_error(SF37KV_EINVAL, "decode_noalloc: %u layers exceed the maximum of %d per call", n,
                         kMaxJobs);
    if ((uint64_t)n * kv_heads > n_counters)
        return set_error(SF37KV_EINVAL,
                         "decode_noalloc: layers x kv_heads = %llu exceeds the %llu split counters",
                         (unsigned long long)n * kv_heads, (unsigned long long)n_counters);
    for (uint32_t i = 0; i < n; i++) {
        const AttnJob &A = jobs[i];
        if (!A.k || !A.v || !A.q || !A.out || A.cap == 0 || A.end < A.start)
            return set_error(SF37KV_EINVAL, "decode_noalloc: layer %u is invalid", i);
    }
    if (n == 0) return SF37KV_OK;
    const uint32_t stride = (G * 130u + 3u) & ~3u;
    const uint64_t cap_parts = part_bytes / ((uint64_t)stride * 4u);
    uint64_t total = 0;
    uint32_t max_rows = 0;
    for (uint32_t i = 0; i < n; i++) {
        total += (uint64_t)(jobs[i].end - jobs[i].start);
        if (jobs[i].end - jobs[i].start > max_rows) max_rows = jobs[i].end - jobs[i].start;
    }
    total *= kv_heads;
    const uint64_t target = (uint64_t)num_sms() * 3 * 8;
    uint64_t per = (total + target - 1) / target;
    if (per < 256) per = 256;
    DecodeParams P;
    P.pdl = 0;
    P.err = nullptr;  // no allocation here (the flag would be allocated on first use)
    for (;;) {
        P.n_jobs = n;
        P.q_heads = q_heads;
        P.kv_heads = kv_heads;
        P.group = G;
        P.part_stride = stride;
        P.qscale = kLog2e / sqrtf(128.0f);
        uint32_t ctas = 0;
        bool any_split = false;
        for (uint32_t i = 0; i < n; i++) {
            const AttnJob &A = jobs[i];
            const uint32_t rows = A.end - A.start;
            uint64_t ns = (rows + per - 1) / per;
            if (ns < 1) ns = 1;
            if (ns > kMaxSplits) ns = kMaxSplits;
            uint32_t sr = (uint32_t)((rows + ns - 1) / ns);
            sr = (sr + 127u) & ~127u;
            if (sr == 0) sr = 128;
            ns = (rows + sr - 1) / sr;
            if (ns < 1) ns = 1;
            if (ns > 1) any_split = true;
            P.job[i] = JobDev{A.k, A.v, A.q, A.gate, A.out, A.start, A.end, A.cap, sr, (uint32_t)ns, ctas,
                              A.k_new, A.v_new, 0};
            ctas += (uint32_t)ns * kv_heads;
        }
        P.total_ctas = ctas;
        if (!any_split || ctas <= cap_parts) break;
        if (per >= max_rows) break;  // cannot happen: one split per layer uses no partials
        per *= 2;
    }
    P.part = part;
    P.counters = counters;
    P.gat = GatherDev{};
    // Counters must start at zero; clear the ones this launch uses.
    if (int rc = check_cuda(cudaMemsetAsync(counters, 0, (size_t)n * kv_heads * 4u, stream),
                            "decode_noalloc counter clear"))
        return rc;
    // The same pipelined kernels as sf37kv_decode's defaults (f16: 4 warps x
    // 3 stages; f32: the bf16 hi/lo tensor-core kernel), without PDL.
    note_stream_appends(stream, P.job, n);
    if (dtype == SF37KV_F16) {
        cudaFuncSetAttribute(decode_f16_pipe_kernel<4, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_pipe(4, 3));
        decode_f16_pipe_kernel<4, 3><<<P.total_ctas, 128, smem_pipe(4, 3), stream>>>(P);
    } else {
        cudaFuncSetAttribute(decode_f32_pipe_kernel<4, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_pipe32(4, 3));
        decode_f32_pipe_kernel<4, 3><<<P.total_ctas, 128, smem_pipe32(4, 3), stream>>>(P);
    }
    g_launches++;
    return check_cuda(cudaGetLastError(), "decode_noalloc launch");
}

}  // namespace sf37kv

namespace sf37kv {

int attention_jobs_gather(const AttnJob *jobs, uint32_t n, uint32_t q_heads, uint32_t kv_heads,
                          uint32_t head_dim, int dtype, cudaStream_t stream, const GatherDev *gat,
                          const uint64_t *offsets) {
    if (n > (uint32_t)kMaxJobs)
        return set_error(SF37KV_EINVAL, "decode_gather: at most %d layers per call", kMaxJobs);
    const uint32_t G = kv_heads ? q_heads / kv_heads : 0;
    if (head_dim != 128 || G == 0 || G > 16)
        return set_error(SF37KV_EUNSUPPORTED, "decode_gather: needs head_dim 128 and group <= 16");
    if (n == 0) return set_error(SF37KV_EINVAL, "decode_gather: no layers (the epoch flag would never rise)");
    for (uint32_t i = 0; i < n; i++) g_gather_off[i] = offsets[i];
    g_gather_cur = gat;
    const int rc = attention_jobs(jobs, n, q_heads, kv_heads, head_dim, dtype, stream);
    g_gather_cur = nullptr;
    return rc;
}

}  // namespace sf37kv
