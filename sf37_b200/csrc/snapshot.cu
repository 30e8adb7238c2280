// Snapshot KV sections: gather (+ int8-grouped encode) and the inverse
// scatter (+ decode), bit-exact with the reference's CUDA-backend formats:
//
//   raw snapshot  (sf37_session_save_snapshot, sf37.c:7298-7320): per
//     position r of a layer, the K row then the V row as f32;
//   disk payload  (sf37_session_save_payload, sf37.c:6980-7010): the same
//     rows, each encoded by payload_encode_kv_row_i8_grouped
//     (sf37.c:6633-6659): per group of `group` elements one f32 scale, then
//     all int8 values.
//
// Position r lives in ring slot (first_pos + r) % cap.  One CTA per encoded
// row; a thread handles 8 consecutive elements (one 16-byte f16 load or two
// f32 loads), so a 64-element group is 8 lanes and its max is 3 shuffles.
// These kernels are HBM- (device buffer) or link- (mapped host buffer) bound.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "kv_internal.cuh"
#include "../../include/sf37_cuda_kv.h"

namespace sf37kv {

extern unsigned long long g_launches;

struct PackJob {
    const void *k, *v;  // caches (unpack writes through them)
    uint32_t cap, first_pos, rows;
    uint64_t offset;    // byte offset of the layer section in the buffer
    uint32_t row_begin; // prefix sum of rows*2 (encoded rows)
};

struct PackParams {
    PackJob job[kMaxJobs];
    uint32_t n_jobs, total_rows;
    uint32_t kv_dim, group, groups;
    uint64_t row_bytes;
    int variant;
};


// Loads 8 consecutive cache elements as f32.
template <typename T>
__device__ __forceinline__ void load8(const T *p, float (&x)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float *p, float (&x)[8]) {
    const float4 a = __ldcs(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldcs(reinterpret_cast<const float4 *>(p) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__half>(const __half *p, float (&x)[8]) {
    const uint4 u = __ldcs(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

template <typename T>
__device__ __forceinline__ void store8(T *p, const float (&x)[8]);
template <>
__device__ __forceinline__ void store8<float>(float *p, const float (&x)[8]) {
    reinterpret_cast<float4 *>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4 *>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
}
template <>
__device__ __forceinline__ void store8<__half>(__half *p, const float (&x)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t *>(&h);
    }
    *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Stores n bytes (n = 8) with the widest stores the address allows.
__device__ __forceinline__ void store_bytes8(uint8_t *dst, uint32_t lo, uint32_t hi) {
    const uintptr_t a = (uintptr_t)dst;
    if ((a & 7u) == 0) {
        *reinterpret_cast<uint2 *>(dst) = make_uint2(lo, hi);
    } else if ((a & 3u) == 0) {
        reinterpret_cast<uint32_t *>(dst)[0] = lo;
        reinterpret_cast<uint32_t *>(dst)[1] = hi;
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) dst[i] = (uint8_t)(lo >> (8 * i));
#pragma unroll
        for (int i = 0; i < 4; i++) dst[4 + i] = (uint8_t)(hi >> (8 * i));
    }
}

// Encodes (FMT) the 8 elements x of row `out` starting at element e0.
template <int FMT>
__device__ __forceinline__ void encode8(const PackParams &P, const float (&x)[8], uint8_t *out, uint32_t e0) {
    if (FMT == SF37KV_FMT_RAW_F32) {
        uint8_t *o = out + (uint64_t)e0 * 4u;
        if (((uintptr_t)o & 15u) == 0) {
            reinterpret_cast<float4 *>(o)[0] = make_float4(x[0], x[1], x[2], x[3]);
            reinterpret_cast<float4 *>(o)[1] = make_float4(x[4], x[5], x[6], x[7]);
        } else {
            for (int i = 0; i < 8; i += 2)
                store_bytes8(o + 4 * i, __float_as_uint(x[i]), __float_as_uint(x[i + 1]));
        }
        return;
    }
    // payload_encode_kv_row_i8_grouped: max |x| over finite values (a NaN or
    // infinite |x| fails the "< inf" test and contributes 0; m >= 0).
    const uint32_t tpg = P.group >> 3;  // threads per group
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float a = fabsf(x[i]);
        m = fmaxf(m, a < INFINITY ? a : 0.f);
    }
    // Groups are whole and lane-aligned, so a lane's partners are active.
    const unsigned act = __activemask();
    for (uint32_t s = 1; s < tpg; s <<= 1) m = fmaxf(m, __shfl_xor_sync(act, m, s));
    float scale, inv;
    if (m > 0.f) {
        if (P.variant == 1) {
            // -ffast-math form: m * (1/127), x * (1/scale), IEEE-rounded.
            scale = __fmul_rn(m, 1.0f / 127.0f);
            inv = __frcp_rn(scale);
        } else {
            scale = __fdiv_rn(m, 127.0f);
            inv = 0.f;
        }
    } else {
        scale = 1.0f;
        inv = 1.0f;
    }
    const uint32_t grp = e0 / P.group;
    if ((threadIdx.x & (tpg - 1u)) == 0) {
        uint8_t *so = out + (uint64_t)grp * 4u;
        const uint32_t u = __float_as_uint(scale);
        if (((uintptr_t)so & 3u) == 0) *reinterpret_cast<uint32_t *>(so) = u;
        else
            for (int i = 0; i < 4; i++) so[i] = (uint8_t)(u >> (8 * i));
    }
    // The reference clamps the code to [-127, 127]; that clamp never fires:
    // every finite v has |v| <= m, so |v * inv| <= 127 (1 + 4 ulp) < 127.5
    // and rint gives at most 127 (likewise for v / scale).  Non-finite v are
    // encoded as 0.  y + 1.5 * 2^23 rounds y to the nearest even integer
    // (as rint), whose two's-complement low byte is the sum's low byte: the
    // int8 code, computed on the FMA pipe rather than the conversion unit.
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float v = fabsf(x[i]) < INFINITY ? x[i] : 0.f;
        const float y = (P.variant == 1 || m <= 0.f) ? __fmul_rn(v, inv) : __fdiv_rn(v, scale);
        q[i] = __float_as_uint(__fadd_rn(y, 12582912.0f));  // rint by 1.5 * 2^23 (|y| <= 127)
    }
    const uint32_t lo = __byte_perm(__byte_perm(q[0], q[1], 0x0040u), __byte_perm(q[2], q[3], 0x0040u), 0x5410u);
    const uint32_t hi = __byte_perm(__byte_perm(q[4], q[5], 0x0040u), __byte_perm(q[6], q[7], 0x0040u), 0x5410u);
    store_bytes8(out + (uint64_t)P.groups * 4u + e0, lo, hi);
}

// Decodes (FMT) the 8 elements of encoded row `in` starting at element e0.
template <int FMT>
__device__ __forceinline__ void decode8(const PackParams &P, const uint8_t *in, uint32_t e0, float (&x)[8]) {
    if (FMT == SF37KV_FMT_RAW_F32) {
        const uint8_t *p = in + (uint64_t)e0 * 4u;
        if (((uintptr_t)p & 15u) == 0) {
            const float4 a = __ldcs(reinterpret_cast<const float4 *>(p));
            const float4 b = __ldcs(reinterpret_cast<const float4 *>(p) + 1);
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
            x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        } else {
            for (int i = 0; i < 8; i++) {
                uint32_t u = 0;
                for (int bb = 0; bb < 4; bb++) u |= (uint32_t)p[4 * i + bb] << (8 * bb);
                x[i] = __uint_as_float(u);
            }
        }
        return;
    }
    // payload_decode_kv_row_i8_grouped (sf37.c:6661-6674): q * scale.
    const uint32_t grp = e0 / P.group;
    const uint8_t *sp = in + (uint64_t)grp * 4u;
    uint32_t su = 0;
    for (int bb = 0; bb < 4; bb++) su |= (uint32_t)sp[bb] << (8 * bb);
    const float scale = __uint_as_float(su);
    const uint8_t *qp = in + (uint64_t)P.groups * 4u + e0;
#pragma unroll
    for (int i = 0; i < 8; i++) x[i] = __fmul_rn((float)(int8_t)qp[i], scale);
}

// Each CTA handles a run of kRowsPerCta encoded rows (row = 2 * position +
// {0: K, 1: V} of a layer section); position r lives at ring slot
// (first_pos + r) % cap.  In the common case (8 * blockDim >= kv_dim) the
// next row's elements are loaded before the current row is encoded.
constexpr uint32_t kRowsPerCta = 16;

struct RowRef {
    uint32_t j, local;
};
__device__ __forceinline__ void advance(const PackParams &P, uint32_t row, RowRef &ref) {
    while (ref.j + 1 < P.n_jobs && P.job[ref.j + 1].row_begin <= row) ref.j++;
    ref.local = row - P.job[ref.j].row_begin;
}

template <typename T>
__device__ __forceinline__ const T *row_src(const PackParams &P, const RowRef &ref) {
    const PackJob &J = P.job[ref.j];
    const uint32_t r = ref.local >> 1, kv = ref.local & 1u;
    const uint64_t slot = (uint64_t)((J.first_pos + r) % J.cap);
    return reinterpret_cast<const T *>(kv ? J.v : J.k) + slot * P.kv_dim;
}

template <typename T, int FMT>
__global__ void __launch_bounds__(128) pack_kernel(uint8_t *dst, const __grid_constant__ PackParams P) {
    const uint32_t row0 = blockIdx.x * kRowsPerCta;
    const uint32_t row1 = min(row0 + kRowsPerCta, P.total_rows);
    RowRef ref{0, 0};
    advance(P, row0, ref);
    const uint32_t e0 = threadIdx.x * 8u;
    if (blockDim.x * 8u >= P.kv_dim) {
        // The CTA's rows are consecutive, so the ring slot advances by one
        // every second row (K, V); one modulo per CTA and per job switch.
        const bool act = e0 < P.kv_dim;
        uint32_t slot = (P.job[ref.j].first_pos + (ref.local >> 1)) % P.job[ref.j].cap;
        auto src_of = [&](const RowRef &c, uint32_t s) {
            const PackJob &J = P.job[c.j];
            return reinterpret_cast<const T *>((c.local & 1u) ? J.v : J.k) + (uint64_t)s * P.kv_dim;
        };
        float x[8];
        if (act) load8<T>(src_of(ref, slot) + e0, x);
        for (uint32_t row = row0; row < row1; row++) {
            const RowRef cur = ref;
            float xn[8];
            if (row + 1 < row1) {
                ref.local++;
                if (ref.local == 2u * P.job[ref.j].rows) {  // next layer section
                    ref.j++;
                    ref.local = 0;
                    slot = P.job[ref.j].first_pos % P.job[ref.j].cap;
                } else if ((ref.local & 1u) == 0) {
                    slot = slot + 1u == P.job[ref.j].cap ? 0u : slot + 1u;
                }
                if (act) load8<T>(src_of(ref, slot) + e0, xn);
            }
            if (act)
                encode8<FMT>(P, x, dst + P.job[cur.j].offset + (uint64_t)cur.local * P.row_bytes, e0);
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = xn[i];
        }
    } else {
        for (uint32_t row = row0; row < row1; row++) {
            advance(P, row, ref);
            const T *src = row_src<T>(P, ref);
            uint8_t *out = dst + P.job[ref.j].offset + (uint64_t)ref.local * P.row_bytes;
            for (uint32_t e = e0; e < P.kv_dim; e += blockDim.x * 8u) {
                float x[8];
                load8<T>(src + e, x);
                encode8<FMT>(P, x, out, e);
            }
        }
    }
}

// Payload rows of the SF37 shape (kv_dim 1024): a thread encodes 16
// elements, so the per-row work (group max, the scale and its IEEE
// reciprocal, addresses) is spread over twice the bytes of pack_kernel.
// A CTA pass handles one position: threads 0-63 its K row, 64-127 its V row
// (a CTA's first row and every section start are even, so the two rows of a
// pass are always the K / V pair of one position).  Same bytes as encode8.
template <typename T>
__device__ __forceinline__ void load16(const T *p, float (&x)[16]) {
    float a[8], b[8];
    load8<T>(p, a);
    load8<T>(p + 8, b);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        x[i] = a[i];
        x[8 + i] = b[i];
    }
}

template <typename T>
__global__ void __launch_bounds__(128) pack_i8x16_kernel(uint8_t *dst, const __grid_constant__ PackParams P) {
    const uint32_t row0 = blockIdx.x * kRowsPerCta;
    const uint32_t row1 = min(row0 + kRowsPerCta, P.total_rows);
    const uint32_t half = threadIdx.x >> 6, t = threadIdx.x & 63u, e0 = t * 16u;
    const uint32_t tpg = P.group >> 4;  // threads per group
    RowRef ref{0, 0};
    advance(P, row0, ref);
    uint32_t slot = (P.job[ref.j].first_pos + (ref.local >> 1)) % P.job[ref.j].cap;
    auto src_of = [&](uint32_t j, uint32_t s) {
        const PackJob &J = P.job[j];
        return reinterpret_cast<const T *>(half ? J.v : J.k) + (uint64_t)s * 1024u + e0;
    };
    float x[16];
    const bool act0 = row0 + half < row1;
    if (act0) load16<T>(src_of(ref.j, slot), x);
    for (uint32_t row = row0; row < row1; row += 2) {
        const uint32_t cj = ref.j, clocal = ref.local;
        const bool act = row + half < row1;
        float xn[16];
        if (row + 2 < row1) {
            ref.local += 2;
            if (ref.local == 2u * P.job[ref.j].rows) {
                ref.j++;
                ref.local = 0;
                slot = P.job[ref.j].first_pos % P.job[ref.j].cap;
            } else {
                slot = slot + 1u == P.job[ref.j].cap ? 0u : slot + 1u;
            }
            if (row + 2 + half < row1) load16<T>(src_of(ref.j, slot), xn);
        }
        if (act) {
            uint8_t *out = dst + P.job[cj].offset + (uint64_t)(clocal + half) * P.row_bytes;
            float m = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const float av = fabsf(x[i]);
                m = fmaxf(m, av < INFINITY ? av : 0.f);
            }
            // a half's 64 threads are two whole warps, active together
            for (uint32_t s = 1; s < tpg; s <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
            float scale, inv;
            if (m > 0.f) {
                if (P.variant == 1) {
                    scale = __fmul_rn(m, 1.0f / 127.0f);
                    inv = __frcp_rn(scale);
                } else {
                    scale = __fdiv_rn(m, 127.0f);
                    inv = 0.f;
                }
            } else {
                scale = 1.0f;
                inv = 1.0f;
            }
            if ((t & (tpg - 1u)) == 0) *reinterpret_cast<float *>(out + (e0 / P.group) * 4u) = scale;
            // as encode8: the reference's [-127, 127] clamp never fires
            uint32_t q[16];
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const float v = fabsf(x[i]) < INFINITY ? x[i] : 0.f;
                const float y = (P.variant == 1 || m <= 0.f) ? __fmul_rn(v, inv) : __fdiv_rn(v, scale);
                // round to nearest even by adding 1.5 * 2^23 (|y| <= 127): the
                // sum's low byte is the int8 code, as rint's would be, and
                // the add runs on the FMA pipe instead of the conversion unit
                q[i] = __float_as_uint(__fadd_rn(y, 12582912.0f));
            }
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; k++)
                w[k] = __byte_perm(__byte_perm(q[4 * k], q[4 * k + 1], 0x0040u),
                                   __byte_perm(q[4 * k + 2], q[4 * k + 3], 0x0040u), 0x5410u);
            uint8_t *qo = out + (uint64_t)P.groups * 4u + e0;
            if (((uintptr_t)qo & 15u) == 0) {
                *reinterpret_cast<uint4 *>(qo) = make_uint4(w[0], w[1], w[2], w[3]);
            } else {
                store_bytes8(qo, w[0], w[1]);
                store_bytes8(qo + 8, w[2], w[3]);
            }
        }
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = xn[i];
    }
}

template <typename T, int FMT>
__global__ void __launch_bounds__(128) unpack_kernel(const uint8_t *src, const __grid_constant__ PackParams P) {
    const uint32_t row0 = blockIdx.x * kRowsPerCta;
    const uint32_t row1 = min(row0 + kRowsPerCta, P.total_rows);
    RowRef ref{0, 0};
    for (uint32_t row = row0; row < row1; row++) {
        advance(P, row, ref);
        T *dst = const_cast<T *>(row_src<T>(P, ref));
        const uint8_t *in = src + P.job[ref.j].offset + (uint64_t)ref.local * P.row_bytes;
        for (uint32_t e0 = threadIdx.x * 8u; e0 < P.kv_dim; e0 += blockDim.x * 8u) {
            float x[8];
            decode8<FMT>(P, in, e0, x);
            store8<T>(dst + e0, x);
        }
    }
}

static uint64_t row_bytes_of(uint32_t kv_dim, int fmt, uint32_t group) {
    if (fmt == SF37KV_FMT_RAW_F32) return (uint64_t)kv_dim * 4u;
    const uint64_t groups = (kv_dim + group - 1u) / group;
    return groups * 4u + kv_dim;
}

static int validate(uint32_t kv_dim, int dtype, int fmt, uint32_t group) {
    if (dtype != SF37KV_F32 && dtype != SF37KV_F16)
        return set_error(SF37KV_EINVAL, "pack: unknown cache dtype %d", dtype);
    if (fmt != SF37KV_FMT_RAW_F32 && fmt != SF37KV_FMT_I8_GROUPED)
        return set_error(SF37KV_EINVAL, "pack: unknown format %d", fmt);
    if (kv_dim == 0 || kv_dim % 8u)
        return set_error(SF37KV_EUNSUPPORTED, "pack: kv_dim %u is not a multiple of 8", kv_dim);
    if (fmt == SF37KV_FMT_I8_GROUPED &&
        (group < 8 || group > 256 || (group & (group - 1u)) || kv_dim % group))
        return set_error(SF37KV_EUNSUPPORTED,
                         "pack: group %u must be a power of two in [8, 256] dividing kv_dim", group);
    return SF37KV_OK;
}

// Launches pack (dir = 0) or unpack (dir = 1) over the layers.
static int launch_layers(void *buf, const sf37kv_pack_layer *layers, uint32_t n, uint32_t kv_dim,
                         int dtype, int fmt, uint32_t group, int variant, int dir,
                         cudaStream_t stream) {
    if (int rc = validate(kv_dim, dtype, fmt, group)) return rc;
    if (!buf && n) return set_error(SF37KV_EINVAL, "pack: buffer is NULL");
    const uint64_t rb = row_bytes_of(kv_dim, fmt, group);
    for (uint32_t base = 0; base < n; base += kMaxJobs) {
        PackParams P;
        P.n_jobs = 0;
        P.kv_dim = kv_dim;
        P.group = fmt == SF37KV_FMT_I8_GROUPED ? group : 8;
        P.groups = fmt == SF37KV_FMT_I8_GROUPED ? kv_dim / group : 0;
        P.row_bytes = rb;
        P.variant = variant;
        uint64_t rows = 0;
        for (uint32_t i = base; i < n && i < base + kMaxJobs; i++) {
            const sf37kv_pack_layer &L = layers[i];
            if (!L.cache.k_cache || !L.cache.v_cache || L.cache.cap == 0)
                return set_error(SF37KV_EINVAL, "pack: layer %u has a null cache or cap 0", i);
            if (L.rows > L.cache.cap)
                return set_error(SF37KV_EINVAL, "pack: layer %u rows %u exceed cap %u", i, L.rows,
                                 L.cache.cap);
            if ((((uintptr_t)L.cache.k_cache | (uintptr_t)L.cache.v_cache) & 15u) != 0)
                return set_error(SF37KV_EINVAL, "pack: layer %u caches must be 16-byte aligned", i);
            if (L.rows == 0) continue;
            PackJob &J = P.job[P.n_jobs++];
            J = PackJob{L.cache.k_cache, L.cache.v_cache, L.cache.cap, L.first_pos, L.rows,
                        L.offset, (uint32_t)rows};
            rows += 2ull * L.rows;
            if (rows > 0x7fffffffull) return set_error(SF37KV_EINVAL, "pack: too many rows");
        }
        if (P.n_jobs == 0) continue;
        P.total_rows = (uint32_t)rows;
        const unsigned grid = (unsigned)((rows + kRowsPerCta - 1) / kRowsPerCta);
        const unsigned threads = kv_dim / 8u < 128u ? ((kv_dim / 8u + 31u) & ~31u) : 128u;
        uint8_t *b = (uint8_t *)buf;
#define SF37_PACK_LAUNCH(T, F)                                                         \
    do {                                                                               \
        if (dir == 0) pack_kernel<T, F><<<grid, threads, 0, stream>>>(b, P);          \
        else unpack_kernel<T, F><<<grid, threads, 0, stream>>>(b, P);                 \
    } while (0)
        // the SF37 shape (1024 elements per row, groups of 16..256) packs
        // payload rows with 16 elements per thread
        bool x16 = dir == 0 && fmt == SF37KV_FMT_I8_GROUPED && kv_dim == 1024u && group >= 16u &&
                   ((uintptr_t)b & 3u) == 0 && P.row_bytes % 4u == 0;
        for (uint32_t i = 0; i < P.n_jobs; i++) x16 = x16 && P.job[i].offset % 4u == 0;
        if (x16) {
            if (dtype == SF37KV_F32) pack_i8x16_kernel<float><<<grid, 128, 0, stream>>>(b, P);
            else pack_i8x16_kernel<__half><<<grid, 128, 0, stream>>>(b, P);
        } else if (dtype == SF37KV_F32) {
            if (fmt == SF37KV_FMT_RAW_F32) SF37_PACK_LAUNCH(float, SF37KV_FMT_RAW_F32);
            else SF37_PACK_LAUNCH(float, SF37KV_FMT_I8_GROUPED);
        } else {
            if (fmt == SF37KV_FMT_RAW_F32) SF37_PACK_LAUNCH(__half, SF37KV_FMT_RAW_F32);
            else SF37_PACK_LAUNCH(__half, SF37KV_FMT_I8_GROUPED);
        }
#undef SF37_PACK_LAUNCH
        g_launches++;
        if (int rc = check_cuda(cudaGetLastError(), dir == 0 ? "pack launch" : "unpack launch"))
            return rc;
    }
    return SF37KV_OK;
}

// ---------------------------------------------------------------- host staging
// Per device: two device staging buffers, two pinned host buffers, a work
// stream and events, created on first use on that device and kept for the
// process (freed by sf37_cuda_cleanup via staging_release()).  A mutex per
// device serializes the pipelines that share them (host threads calling
// concurrently on one device wait for each other).
constexpr uint64_t kStageBytes = 64ull << 20;
struct Staging {
    bool ready = false, host_ready = false;
    void *stage[2] = {nullptr, nullptr};
    cudaStream_t copy = nullptr, work = nullptr;
    cudaEvent_t ev_packed[2], ev_copied[2], ev_start;
    void *hbuf[2] = {nullptr, nullptr};
    cudaEvent_t ev_host[2];
    std::mutex mu;
};
constexpr int kMaxStagingDevices = 64;
static Staging g_staging[kMaxStagingDevices];

// The current device's staging set (not yet initialized).
static int current_staging(Staging **out) {
    int dev = 0;
    if (int rc = check_cuda(cudaGetDevice(&dev), "staging get device")) return rc;
    if (dev < 0 || dev >= kMaxStagingDevices)
        return set_error(SF37KV_EUNSUPPORTED, "staging: device %d out of range", dev);
    *out = &g_staging[dev];
    return SF37KV_OK;
}

static int staging_init(Staging &S) {
    if (S.ready) return SF37KV_OK;
    for (int i = 0; i < 2; i++)
        if (int rc = check_cuda(cudaMalloc(&S.stage[i], kStageBytes), "staging alloc")) return rc;
    if (int rc = check_cuda(cudaStreamCreateWithFlags(&S.copy, cudaStreamNonBlocking), "stream")) return rc;
    if (int rc = check_cuda(cudaStreamCreateWithFlags(&S.work, cudaStreamNonBlocking), "stream")) return rc;
    for (int i = 0; i < 2; i++) {
        cudaEventCreateWithFlags(&S.ev_packed[i], cudaEventDisableTiming);
        cudaEventCreateWithFlags(&S.ev_copied[i], cudaEventDisableTiming);
    }
    cudaEventCreateWithFlags(&S.ev_start, cudaEventDisableTiming);
    if (int rc = check_cuda(cudaGetLastError(), "staging events")) return rc;
    S.ready = true;
    return SF37KV_OK;
}

// Splits each layer's section into chunks of at most kStageBytes and runs
// pack -> D2H (dir 0) or H2D -> unpack (dir 1) with double buffering.
static int host_pipeline(void *host, const sf37kv_pack_layer *layers, uint32_t n, uint32_t kv_dim,
                         int dtype, int fmt, uint32_t group, int variant, int dir) {
    if (int rc = validate(kv_dim, dtype, fmt, group)) return rc;
    if (!host && n) return set_error(SF37KV_EINVAL, "pack: host buffer is NULL");
    Staging *SP = nullptr;
    if (int rc = current_staging(&SP)) return rc;
    Staging &S = *SP;
    std::lock_guard<std::mutex> lk(S.mu);
    if (int rc = staging_init(S)) return rc;
    const uint64_t rb = row_bytes_of(kv_dim, fmt, group);
    const uint64_t chunk_rows = kStageBytes / (2 * rb);
    if (chunk_rows == 0) return set_error(SF37KV_EUNSUPPORTED, "pack: row larger than staging");
    // Order after everything already queued on the library stream.
    cudaEventRecord(S.ev_start, current_stream());
    cudaStreamWaitEvent(S.work, S.ev_start, 0);
    cudaStreamWaitEvent(S.copy, S.ev_start, 0);
    int buf = 0;
    bool used[2] = {false, false};
    for (uint32_t i = 0; i < n; i++) {
        const sf37kv_pack_layer &L = layers[i];
        for (uint64_t r0 = 0; r0 < L.rows; r0 += chunk_rows) {
            const uint32_t nr = (uint32_t)((L.rows - r0) < chunk_rows ? (L.rows - r0) : chunk_rows);
            sf37kv_pack_layer c = L;
            c.first_pos = L.first_pos + (uint32_t)r0;
            c.rows = nr;
            c.offset = 0;
            const uint64_t bytes = 2ull * nr * rb;
            uint8_t *h = (uint8_t *)host + L.offset + 2ull * r0 * rb;
            if (dir == 0) {
                if (used[buf]) cudaStreamWaitEvent(S.work, S.ev_copied[buf], 0);
                if (int rc = launch_layers(S.stage[buf], &c, 1, kv_dim, dtype, fmt, group, variant, 0,
                                           S.work))
                    return rc;
                cudaEventRecord(S.ev_packed[buf], S.work);
                cudaStreamWaitEvent(S.copy, S.ev_packed[buf], 0);
                if (int rc = check_cuda(cudaMemcpyAsync(h, S.stage[buf], bytes, cudaMemcpyDeviceToHost,
                                                        S.copy), "pack D2H"))
                    return rc;
                cudaEventRecord(S.ev_copied[buf], S.copy);
            } else {
                if (used[buf]) cudaStreamWaitEvent(S.copy, S.ev_packed[buf], 0);
                if (int rc = check_cuda(cudaMemcpyAsync(S.stage[buf], h, bytes, cudaMemcpyHostToDevice,
                                                        S.copy), "unpack H2D"))
                    return rc;
                cudaEventRecord(S.ev_copied[buf], S.copy);
                cudaStreamWaitEvent(S.work, S.ev_copied[buf], 0);
                if (int rc = launch_layers(S.stage[buf], &c, 1, kv_dim, dtype, fmt, group, variant, 1,
                                           S.work))
                    return rc;
                cudaEventRecord(S.ev_packed[buf], S.work);
            }
            used[buf] = true;
            buf ^= 1;
        }
    }
    if (int rc = check_cuda(cudaStreamSynchronize(S.copy), "pack copy sync")) return rc;
    if (int rc = check_cuda(cudaStreamSynchronize(S.work), "pack work sync")) return rc;
    // Later work on the library stream must see restored caches.
    return SF37KV_OK;
}

// ---------------------------------------------------------------- streams
// Packed bytes to / from a host callback (a file descriptor, a socket) in
// chunks of at most kStageBytes, through two pinned host buffers: the device
// packs and copies chunk c while the host consumes chunk c-1 (pack), or the
// host produces chunk c while the device copies in and unpacks chunk c-1
// (unpack).  A chunk is a run of whole rows of one or more consecutive layer
// sections, so the callback sees the sections' bytes in order.
static int host_buffers_init(Staging &S) {
    if (int rc = staging_init(S)) return rc;
    if (S.host_ready) return SF37KV_OK;
    for (int i = 0; i < 2; i++) {
        if (int rc = check_cuda(cudaHostAlloc(&S.hbuf[i], kStageBytes, cudaHostAllocDefault), "pinned stream buffer"))
            return rc;
        if (int rc = check_cuda(cudaEventCreateWithFlags(&S.ev_host[i], cudaEventDisableTiming), "event")) return rc;
    }
    S.host_ready = true;
    return SF37KV_OK;
}

namespace {
struct Chunk {
    sf37kv_pack_layer piece[kMaxJobs];
    uint32_t layer[kMaxJobs];   // index of the piece's layer section
    uint32_t row0[kMaxJobs];    // its first row within that section
    uint32_t n = 0;
    uint64_t bytes = 0;
};

// Cuts the layer sections into chunks of whole rows, each <= cap_bytes.
struct Chunker {
    const sf37kv_pack_layer *layers;
    uint32_t n_layers, li = 0;
    uint64_t r0 = 0, rb, cap_rows;
    bool next(Chunk *c) {
        c->n = 0;
        c->bytes = 0;
        uint64_t room = cap_rows;
        while (li < n_layers && room > 0 && c->n < (uint32_t)kMaxJobs) {
            const sf37kv_pack_layer &L = layers[li];
            const uint64_t left = L.rows - r0;
            if (left == 0) {
                li++;
                r0 = 0;
                continue;
            }
            const uint64_t take = left < room ? left : room;
            sf37kv_pack_layer p = L;
            p.first_pos = L.first_pos + (uint32_t)r0;
            p.rows = (uint32_t)take;
            p.offset = c->bytes;
            c->layer[c->n] = li;
            c->row0[c->n] = (uint32_t)r0;
            c->piece[c->n++] = p;
            c->bytes += 2ull * take * rb;
            room -= take;
            r0 += take;
            if (r0 == L.rows) {
                li++;
                r0 = 0;
            }
        }
        return c->n > 0;
    }
};
}  // namespace

int pack_stream(const sf37kv_pack_layer *layers, uint32_t n, uint32_t kv_dim, int dtype, int fmt,
                uint32_t group, int (*sink)(const void *, uint64_t, void *), void *ctx) {
    if (int rc = validate(kv_dim, dtype, fmt, group)) return rc;
    Staging *SP = nullptr;
    if (int rc = current_staging(&SP)) return rc;
    Staging &S = *SP;
    std::lock_guard<std::mutex> lk(S.mu);
    if (int rc = host_buffers_init(S)) return rc;
    const uint64_t rb = row_bytes_of(kv_dim, fmt, group);
    Chunker ck{layers, n, 0, 0, rb, kStageBytes / (2 * rb)};
    if (ck.cap_rows == 0) return set_error(SF37KV_EUNSUPPORTED, "pack: row larger than staging");
    cudaEventRecord(S.ev_start, current_stream());
    cudaStreamWaitEvent(S.work, S.ev_start, 0);
    Chunk c;
    uint64_t pending[2] = {0, 0};
    int b = 0, rc = SF37KV_OK;
    bool have_prev = false;
    while (rc == SF37KV_OK && ck.next(&c)) {
        // buffer b was consumed by the host before the previous iteration ended
        rc = launch_layers(S.stage[b], c.piece, c.n, kv_dim, dtype, fmt, group, 1, 0, S.work);
        if (!rc) rc = check_cuda(cudaMemcpyAsync(S.hbuf[b], S.stage[b], c.bytes, cudaMemcpyDeviceToHost,
                                                 S.work), "stream D2H");
        if (!rc) rc = check_cuda(cudaEventRecord(S.ev_host[b], S.work), "event");
        pending[b] = c.bytes;
        if (!rc && have_prev) {
            rc = check_cuda(cudaEventSynchronize(S.ev_host[b ^ 1]), "stream sync");
            if (!rc && sink(S.hbuf[b ^ 1], pending[b ^ 1], ctx)) rc = SF37KV_EINVAL;
        }
        have_prev = true;
        b ^= 1;
    }
    if (!rc && have_prev) {
        rc = check_cuda(cudaEventSynchronize(S.ev_host[b ^ 1]), "stream sync");
        if (!rc && sink(S.hbuf[b ^ 1], pending[b ^ 1], ctx)) rc = SF37KV_EINVAL;
    }
    (void)cudaStreamSynchronize(S.work);
    return rc;
}

int unpack_stream(const sf37kv_pack_layer *layers, uint32_t n, uint32_t kv_dim, int dtype, int fmt,
                  uint32_t group, int (*source)(void *, uint64_t, void *), void *ctx) {
    if (int rc = validate(kv_dim, dtype, fmt, group)) return rc;
    Staging *SP = nullptr;
    if (int rc = current_staging(&SP)) return rc;
    Staging &S = *SP;
    std::lock_guard<std::mutex> lk(S.mu);
    if (int rc = host_buffers_init(S)) return rc;
    const uint64_t rb = row_bytes_of(kv_dim, fmt, group);
    Chunker ck{layers, n, 0, 0, rb, kStageBytes / (2 * rb)};
    if (ck.cap_rows == 0) return set_error(SF37KV_EUNSUPPORTED, "pack: row larger than staging");
    cudaEventRecord(S.ev_start, current_stream());
    cudaStreamWaitEvent(S.work, S.ev_start, 0);
    Chunk c;
    int b = 0, rc = SF37KV_OK;
    bool used[2] = {false, false};
    while (rc == SF37KV_OK && ck.next(&c)) {
        // the H2D copy of chunk c-2 out of this host buffer must be done
        if (used[b]) rc = check_cuda(cudaEventSynchronize(S.ev_host[b]), "stream sync");
        if (!rc && source(S.hbuf[b], c.bytes, ctx)) rc = SF37KV_EINVAL;
        if (!rc) rc = check_cuda(cudaMemcpyAsync(S.stage[b], S.hbuf[b], c.bytes, cudaMemcpyHostToDevice,
                                                 S.work), "stream H2D");
        if (!rc) rc = check_cuda(cudaEventRecord(S.ev_host[b], S.work), "event");
        if (!rc) rc = launch_layers(S.stage[b], c.piece, c.n, kv_dim, dtype, fmt, group, 1, 1, S.work);
        used[b] = true;
        b ^= 1;
    }
    const int rs = check_cuda(cudaStreamSynchronize(S.work), "stream sync");
    return rc ? rc : rs;
}

// ---------------------------------------------------------------- KV-head slices
// A GPU that holds KV heads [h0, h0 + n) of every layer writes (reads) only
// its columns of the full-width record rows: elements [col0, col0 + kv_dim)
// of each full_kv_dim-element row.  The device packs the slice compactly
// (kv_dim-wide rows) into the staging buffer; the host then scatters each
// row's pieces into the full layout (raw: one run of 4 kv_dim bytes; payload:
// the slice's group scales and its codes), so no byte of another slice is
// touched and several GPUs can fill one record buffer.
namespace {
struct SliceGeom {
    uint32_t kv_dim, full, col0, group;
    int fmt;
    uint64_t rb, rbf;  // compact and full row bytes
    // (offset, length) of the slice's pieces within a compact / full row
    uint32_t n_pieces() const { return fmt == SF37KV_FMT_RAW_F32 ? 1u : 2u; }
    void piece(uint32_t k, uint64_t &src, uint64_t &dst, uint64_t &len) const {
        if (fmt == SF37KV_FMT_RAW_F32) {
            src = 0;
            dst = (uint64_t)col0 * 4u;
            len = (uint64_t)kv_dim * 4u;
        } else if (k == 0) {  // group scales
            src = 0;
            dst = (uint64_t)(col0 / group) * 4u;
            len = (uint64_t)(kv_dim / group) * 4u;
        } else {  // int8 codes
            src = (uint64_t)(kv_dim / group) * 4u;
            dst = (uint64_t)(full / group) * 4u + col0;
            len = kv_dim;
        }
    }
};

// Copies the pieces of every row of chunk c between the compact staging
// image `compact` and the full-layout host buffer, with a few threads.
void scatter_gather(const Chunk &c, const sf37kv_pack_layer *layers, const SliceGeom &G, uint8_t *compact,
                    uint8_t *host, bool to_host) {
    uint64_t total_rows = 0;
    for (uint32_t i = 0; i < c.n; i++) total_rows += 2ull * c.piece[i].rows;
    auto work = [&](uint64_t lo, uint64_t hi) {
        uint64_t base = 0;
        for (uint32_t i = 0; i < c.n && base < hi; i++) {
            const uint64_t nr = 2ull * c.piece[i].rows;
            const uint64_t a = lo > base ? lo - base : 0, b = hi - base < nr ? hi - base : nr;
            for (uint64_t r = a; r < b; r++) {
                uint8_t *cr = compact + c.piece[i].offset + r * G.rb;
                uint8_t *hr = host + layers[c.layer[i]].offset + (2ull * c.row0[i] + r) * G.rbf;
                for (uint32_t k = 0; k < G.n_pieces(); k++) {
                    uint64_t so, dof, len;
                    G.piece(k, so, dof, len);
                    if (to_host) memcpy(hr + dof, cr + so, len);
                    else memcpy(cr + so, hr + dof, len);
                }
            }
            base += nr;
        }
    };
    unsigned nt = std::thread::hardware_concurrency();
    nt = nt < 1 ? 1 : nt > 8 ? 8 : nt;
    if (total_rows < 4096) nt = 1;
    std::vector<std::thread> th;
    for (unsigned t = 1; t < nt; t++)
        th.emplace_back(work, total_rows * t / nt, total_rows * (t + 1) / nt);
    work(0, total_rows / nt);
    for (auto &x : th) x.join();
}
}  // namespace

static int slice_pipeline(void *host, const sf37kv_pack_layer *layers, uint32_t n, uint32_t kv_dim,
                          uint32_t full_kv_dim, uint32_t col0, int dtype, int fmt, uint32_t group, int variant,
                          int dir) {
    if (int rc = validate(kv_dim, dtype, fmt, group)) return rc;
    if (int rc = validate(full_kv_dim, dtype, fmt, group)) return rc;
    if (!host && n) return set_error(SF37KV_EINVAL, "pack slice: host buffer is NULL");
    if (col0 % 8u || (uint64_t)col0 + kv_dim > full_kv_dim ||
        (fmt == SF37KV_FMT_I8_GROUPED && col0 % group))
        return set_error(SF37KV_EINVAL, "pack slice: columns [%u, %u) do not fit %u (payload: group-aligned)", col0,
                         col0 + kv_dim, full_kv_dim);
    Staging *SP = nullptr;
    if (int rc = current_staging(&SP)) return rc;
    Staging &S = *SP;
    std::lock_guard<std::mutex> lk(S.mu);
    if (int rc = host_buffers_init(S)) return rc;
    SliceGeom G{kv_dim, full_kv_dim, col0, group, fmt, row_bytes_of(kv_dim, fmt, group),
                row_bytes_of(full_kv_dim, fmt, group)};
    Chunker ck{layers, n, 0, 0, G.rb, kStageBytes / (2 * G.rb)};
    cudaEventRecord(S.ev_start, current_stream());
    cudaStreamWaitEvent(S.work, S.ev_start, 0);
    uint8_t *h = (uint8_t *)host;
    Chunk c[2];
    int b = 0, rc = SF37KV_OK;
    bool have_prev = false, used[2] = {false, false};
    while (rc == SF37KV_OK && ck.next(&c[b])) {
        if (dir == 0) {
            rc = launch_layers(S.stage[b], c[b].piece, c[b].n, kv_dim, dtype, fmt, group, variant, 0, S.work);
            if (!rc) rc = check_cuda(cudaMemcpyAsync(S.hbuf[b], S.stage[b], c[b].bytes, cudaMemcpyDeviceToHost,
                                                     S.work), "slice D2H");
            if (!rc) rc = check_cuda(cudaEventRecord(S.ev_host[b], S.work), "event");
            if (!rc && have_prev) {  // scatter the previous chunk while this one packs
                rc = check_cuda(cudaEventSynchronize(S.ev_host[b ^ 1]), "slice sync");
                if (!rc) scatter_gather(c[b ^ 1], layers, G, (uint8_t *)S.hbuf[b ^ 1], h, true);
            }
        } else {
            if (used[b]) rc = check_cuda(cudaEventSynchronize(S.ev_host[b]), "slice sync");
            if (!rc) scatter_gather(c[b], layers, G, (uint8_t *)S.hbuf[b], h, false);
            if (!rc) rc = check_cuda(cudaMemcpyAsync(S.stage[b], S.hbuf[b], c[b].bytes, cudaMemcpyHostToDevice,
                                                     S.work), "slice H2D");
            if (!rc) rc = check_cuda(cudaEventRecord(S.ev_host[b], S.work), "event");
            if (!rc) rc = launch_layers(S.stage[b], c[b].piece, c[b].n, kv_dim, dtype, fmt, group, 1, 1, S.work);
            used[b] = true;
        }
        have_prev = true;
        b ^= 1;
    }
    if (!rc && dir == 0 && have_prev) {
        rc = check_cuda(cudaEventSynchronize(S.ev_host[b ^ 1]), "slice sync");
        if (!rc) scatter_gather(c[b ^ 1], layers, G, (uint8_t *)S.hbuf[b ^ 1], h, true);
    }
    const int rs = check_cuda(cudaStreamSynchronize(S.work), "slice sync");
    return rc ? rc : rs;
}

void staging_release() {
    for (Staging &S : g_staging) {
        std::lock_guard<std::mutex> lk(S.mu);
        for (int i = 0; i < 2; i++) {
            if (S.stage[i]) cudaFree(S.stage[i]);
            S.stage[i] = nullptr;
            if (S.hbuf[i]) {
                cudaFreeHost(S.hbuf[i]);
                cudaEventDestroy(S.ev_host[i]);
            }
            S.hbuf[i] = nullptr;
        }
        S.ready = S.host_ready = false;
    }
}

}  // namespace sf37kv

using namespace sf37kv;

extern "C" uint64_t sf37kv_row_bytes(uint32_t kv_dim, int fmt, uint32_t group) {
    return row_bytes_of(kv_dim, fmt, group);
}

extern "C" int sf37kv_pack(void *dst, const sf37kv_pack_layer *layers, uint32_t n_layers,
                           uint32_t kv_dim, int dtype, int fmt, uint32_t group, int variant,
                           void *stream) {
    return launch_layers(dst, layers, n_layers, kv_dim, dtype, fmt, group, variant, 0,
                         stream ? (cudaStream_t)stream : current_stream());
}

extern "C" int sf37kv_unpack(const void *src, const sf37kv_pack_layer *layers, uint32_t n_layers,
                             uint32_t kv_dim, int dtype, int fmt, uint32_t group, void *stream) {
    return launch_layers(const_cast<void *>(src), layers, n_layers, kv_dim, dtype, fmt, group, 1, 1,
                         stream ? (cudaStream_t)stream : current_stream());
}

extern "C" int sf37kv_pack_to_host(void *host_dst, const sf37kv_pack_layer *layers, uint32_t n_layers,
                                   uint32_t kv_dim, int dtype, int fmt, uint32_t group, int variant) {
    return host_pipeline(host_dst, layers, n_layers, kv_dim, dtype, fmt, group, variant, 0);
}

extern "C" int sf37kv_pack_slice_to_host(void *host_dst, const sf37kv_pack_layer *layers, uint32_t n_layers,
                                         uint32_t kv_dim, uint32_t full_kv_dim, uint32_t col0, int dtype, int fmt,
                                         uint32_t group, int variant) {
    return slice_pipeline(host_dst, layers, n_layers, kv_dim, full_kv_dim, col0, dtype, fmt, group, variant, 0);
}

extern "C" int sf37kv_unpack_slice_from_host(const void *host_src, const sf37kv_pack_layer *layers,
                                             uint32_t n_layers, uint32_t kv_dim, uint32_t full_kv_dim, uint32_t col0,
                                             int dtype, int fmt, uint32_t group) {
    return slice_pipeline(const_cast<void *>(host_src), layers, n_layers, kv_dim, full_kv_dim, col0, dtype, fmt,
                          group, 1, 1);
}

extern "C" int sf37kv_unpack_from_host(const void *host_src, const sf37kv_pack_layer *layers,
                                       uint32_t n_layers, uint32_t kv_dim, int dtype, int fmt,
                                       uint32_t group) {
    return host_pipeline(const_cast<void *>(host_src), layers, n_layers, kv_dim, dtype, fmt, group, 1,
                         1);
}

// ---------------------------------------------------------------- drop-in
static int dropin_pack(void *host, const sf37_cuda_tensor *k, const sf37_cuda_tensor *v,
                       uint32_t first_pos, uint32_t rows, uint32_t cap, uint32_t kv_dim, int fmt,
                       uint32_t group, int variant, int dir, const char *what) {
    if (!host || !k || !v || cap == 0 || kv_dim == 0 || rows > cap) return 0;
    const uint64_t need = (uint64_t)cap * kv_dim * 4u;
    if (k->bytes < need || v->bytes < need) return 0;
    sf37kv_pack_layer L;
    memset(&L, 0, sizeof(L));
    L.cache.k_cache = k->ptr;
    L.cache.v_cache = v->ptr;
    L.cache.cap = cap;
    L.first_pos = first_pos;
    L.rows = rows;
    L.offset = 0;
    if (host_pipeline(host, &L, 1, kv_dim, SF37KV_F32, fmt, group, variant, dir)) {
        fprintf(stderr, "sf37: %s failed: %s\n", what, sf37kv_last_error());
        return 0;
    }
    return 1;
}

extern "C" int sf37_cuda_kv_pack_rows_f32(void *host_dst, const sf37_cuda_tensor *k_cache,
                                          const sf37_cuda_tensor *v_cache, uint32_t first_pos,
                                          uint32_t rows, uint32_t cache_cap, uint32_t kv_dim) {
    return dropin_pack(host_dst, k_cache, v_cache, first_pos, rows, cache_cap, kv_dim,
                       SF37KV_FMT_RAW_F32, 64, 1, 0, "kv pack f32");
}

extern "C" int sf37_cuda_kv_unpack_rows_f32(const void *host_src, sf37_cuda_tensor *k_cache,
                                            sf37_cuda_tensor *v_cache, uint32_t first_pos,
                                            uint32_t rows, uint32_t cache_cap, uint32_t kv_dim) {
    return dropin_pack(const_cast<void *>(host_src), k_cache, v_cache, first_pos, rows, cache_cap,
                       kv_dim, SF37KV_FMT_RAW_F32, 64, 1, 1, "kv unpack f32");
}

extern "C" int sf37_cuda_kv_pack_rows_i8g(void *host_dst, const sf37_cuda_tensor *k_cache,
                                          const sf37_cuda_tensor *v_cache, uint32_t first_pos,
                                          uint32_t rows, uint32_t cache_cap, uint32_t kv_dim,
                                          uint32_t group, int variant) {
    return dropin_pack(host_dst, k_cache, v_cache, first_pos, rows, cache_cap, kv_dim,
                       SF37KV_FMT_I8_GROUPED, group, variant, 0, "kv pack i8g");
}

extern "C" int sf37_cuda_kv_unpack_rows_i8g(const void *host_src, sf37_cuda_tensor *k_cache,
                                            sf37_cuda_tensor *v_cache, uint32_t first_pos,
                                            uint32_t rows, uint32_t cache_cap, uint32_t kv_dim,
                                            uint32_t group) {
    return dropin_pack(const_cast<void *>(host_src), k_cache, v_cache, first_pos, rows, cache_cap,
                       kv_dim, SF37KV_FMT_I8_GROUPED, group, 1, 1, "kv unpack i8g");
}
