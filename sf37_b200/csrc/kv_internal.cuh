// Internal declarations shared by the libsf37kv translation units.
//
// Layout of every KV cache on the device: [cap][kv_heads][head_dim] with
// element type f32 (the reference's only type, sf37.c:2033-2043,
// sf37_cuda.cu:2408-2990) or f16 (the B200 throughput mode).  A "row" is one
// position: kv_heads*head_dim contiguous elements.  Logical position r lives
// in physical slot r % cap (sf37_cuda.cu:6368, 2762).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/sf37kv.h"

namespace sf37kv {

constexpr int kMaxJobs = 64;       // jobs (layers or queries) per launch
constexpr int kHeadDim = 128;      // head_dim of the fast kernels

// ---------------------------------------------------------------- errors
// Records a formatted message as the thread's last error and returns code.
int set_error(int code, const char *fmt, ...);
// Returns SF37KV_OK if err == cudaSuccess, else records and returns ECUDA.
int check_cuda(cudaError_t err, const char *what);

cudaStream_t current_stream();
int *device_error_flag();
int num_sms();

// ---------------------------------------------------------------- scratch
// Grow-only device scratch for split-K partials plus a zeroed counter array
// (self-resetting: the last CTA of each group puts its counter back to 0).
struct Scratch {
    float *part = nullptr;       // partial O and (m, l) per CTA
    uint64_t part_bytes = 0;
    uint32_t *counters = nullptr;
    uint64_t n_counters = 0;
};
int scratch_get(uint64_t part_bytes, uint64_t n_counters, Scratch *out);
void scratch_release();
void staging_release();  // snapshot staging buffers

// Snapshot sections streamed through pinned chunks to / from a host callback
// (returns nonzero to stop; the call then fails with SF37KV_EINVAL and the
// callback's own message stays the last error).  Synchronous.
int pack_stream(const sf37kv_pack_layer *layers, uint32_t n, uint32_t kv_dim, int dtype, int fmt,
                uint32_t group, int (*sink)(const void *, uint64_t, void *), void *ctx);
int unpack_stream(const sf37kv_pack_layer *layers, uint32_t n, uint32_t kv_dim, int dtype, int fmt,
                  uint32_t group, int (*source)(void *, uint64_t, void *), void *ctx);

// ---------------------------------------------------------------- attention
// One attention "job": one query vector set (q_heads heads) over logical
// rows [start, end) of one cache.  A decode layer is one job; a prefill token
// on the fallback path is one job.
struct AttnJob {
    const void *k;
    const void *v;
    const float *q;       // [q_heads][head_dim] f32
    const float *gate;    // [q_heads] f32 or nullptr (gate factor 1)
    float *out;           // [q_heads][head_dim] f32
    uint32_t start, end;  // logical rows
    uint32_t cap;
    // Optional row appended at position end-1 before attention (f32
    // [kv_heads*head_dim]); the fast kernels store it themselves.
    const float *k_new = nullptr, *v_new = nullptr;
    // Optional q/k head preparation (RMS norm + RoPE) applied in the kernel
    // to q and k_new before use (sf37kv_decode_prep).
    const sf37kv_qk_prep *prep = nullptr;
};

// Launches attention for n jobs (any n; chunked internally).
// dtype: SF37KV_F32 or SF37KV_F16.  Writes out = softmax(qK^T/sqrt(d))V *
// sigmoid(gate) per head; an empty row range writes zeros.
int attention_jobs(const AttnJob *jobs, uint32_t n, uint32_t q_heads, uint32_t kv_heads,
                   uint32_t head_dim, int dtype, cudaStream_t stream);

// The same split-K decode with caller-provided partials and counters; never
// allocates (see decode_noalloc.cu).
int attention_jobs_prealloc(const AttnJob *jobs, uint32_t n, uint32_t q_heads, uint32_t kv_heads,
                            uint32_t head_dim, int dtype, cudaStream_t stream, float *part,
                            uint64_t part_bytes, uint32_t *counters, uint64_t n_counters);

// Peer-memory output gather (multi-GPU): every final output value is also
// stored into the gather buffer of each other rank (plain stores over
// NVLink); the last group to finish on this GPU raises this rank's epoch flag
// in every rank's flag array (system-scope release).  world == 0: disabled.
struct GatherDev {
    float *peer[8];
    uint32_t *peer_flags[8];
    uint32_t world, rank, epoch, total_groups;
    uint32_t *done;  // groups finished in this launch (self-resetting)
};

// Validates a peer descriptor and fills the device form (gather.cu).
int gather_dev(const sf37kv_peer_gather *g, uint32_t epoch, GatherDev *d);

int attention_jobs_gather(const AttnJob *jobs, uint32_t n, uint32_t q_heads, uint32_t kv_heads,
                          uint32_t head_dim, int dtype, cudaStream_t stream, const GatherDev *gat,
                          const uint64_t *offsets);

// Logical start row of the query at position pos (sf37_cuda.cu:2752-2758).
static inline uint32_t start_at(uint32_t pos, uint32_t cap, int sliding, uint32_t window) {
    const uint32_t have = pos + 1u;
    uint32_t start = 0;
    if (have > cap) start = have - cap;
    if (sliding && have > window) {
        const uint32_t sw = have - window;
        if (sw > start) start = sw;
    }
    return start;
}

// ---------------------------------------------------------------- append
struct AppendJob {
    void *k_cache, *v_cache;
    const float *k, *v;   // [n_tok][kv_dim] f32
    uint32_t pos0, n_tok, cap;
};
int append_jobs(const AppendJob *jobs, uint32_t n, uint32_t kv_dim, int dtype,
                cudaStream_t stream);

// ---------------------------------------------------------------- small device helpers
__device__ __forceinline__ float sigmoid_dev(float x) {
    // sf37_sigmoid (sf37_ops.c:9-16): the numerically safe two-branch form.
    if (x >= 0.0f) {
        const float z = expf(-x);
        return 1.0f / (1.0f + z);
    }
    const float z = expf(x);
    return z / (1.0f + z);
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

}  // namespace sf37kv
