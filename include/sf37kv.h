/*
 * Native C ABI of libsf37kv: the B200 KV-cache hot path beyond the
 * reference's fp32 drop-in entry points (sf37_cuda_kv.h).
 *
 * Adds what the reference ABI cannot express:
 *   - f16 caches (the throughput mode; the reference caches are f32 only),
 *   - multi-layer batched calls (one launch for many independent layers),
 *   - explicit CUDA streams (passed as void*, NULL = the library stream),
 *   - error codes plus sf37kv_last_error() instead of stderr-only failures,
 *   - bf16 queries for chunked prefill,
 *   - KV-head slices for the multi-GPU layout (a GPU that owns heads
 *     [h0, h0+n) of every layer simply passes kv_heads = n and its slice of
 *     the queries: see sf37kv_decode()).
 *
 * All pointers are device pointers unless named host_*; all sizes are
 * element counts unless named *_bytes.  Every call is asynchronous on its
 * stream unless documented otherwise.
 */
#ifndef SF37KV_H
#define SF37KV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SF37KV_OK = 0,
    SF37KV_EINVAL = 1,       /* bad argument; nothing was launched */
    SF37KV_ECUDA = 2,        /* a CUDA call failed */
    SF37KV_ENOMEM = 3,       /* device or host allocation failed */
    SF37KV_EUNSUPPORTED = 4  /* valid but not implemented shape */
};

/* Cache element type = element size in bytes. */
enum { SF37KV_F16 = 2, SF37KV_F32 = 4 };
/* Query element type for prefill. */
enum { SF37KV_Q_F32 = 0, SF37KV_Q_BF16 = 1 };
/* Snapshot KV row formats. */
enum { SF37KV_FMT_RAW_F32 = 0, SF37KV_FMT_I8_GROUPED = 1 };

const char *sf37kv_last_error(void);
const char *sf37kv_version(void);

/* Library stream used by the drop-in entry points and by native calls given
 * stream == NULL.  Default: the legacy default stream (as the reference). */
int sf37kv_set_stream(void *stream);
void *sf37kv_get_stream(void);

/* One layer's cache.  k_cache/v_cache: [cap][kv_heads][head_dim] of dtype.
 * Positions live in ring slot pos % cap.  sliding layers attend to the
 * last `window` positions (sf37_cuda.cu:2752-2758). */
typedef struct {
    void *k_cache;
    void *v_cache;
    uint32_t cap;
    uint32_t sliding;
    uint32_t window;
    uint32_t reserved;
} sf37kv_cache;

/* One layer of a decode step. */
typedef struct {
    sf37kv_cache cache;
    uint32_t pos;          /* position of this token */
    uint32_t reserved;
    const float *q;        /* [q_heads][head_dim] */
    const float *gate;     /* [q_heads] or NULL (no gate) */
    float *out;            /* [q_heads][head_dim] */
    const float *k_new;    /* [kv_heads*head_dim] row appended at pos, or NULL */
    const float *v_new;
} sf37kv_decode_layer;

/* Decode step over n_layers independent layers: for each layer, append
 * (k_new, v_new) at slot pos % cap (f32 -> f16 round-to-nearest-even for f16
 * caches) when k_new is non-NULL, then GQA attention of the query at pos:
 * out[h] = softmax(q[h] K^T / sqrt(head_dim)) V * sigmoid(gate[h]), with
 * K/V head h / (q_heads/kv_heads) (sf37_cuda.cu:3079-3161 semantics).
 * head_dim 128 and q_heads/kv_heads <= 16 use the fast kernels; other shapes
 * use a generic kernel (head_dim <= 256). */
int sf37kv_decode(const sf37kv_decode_layer *layers, uint32_t n_layers,
                  uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                  int dtype, void *stream);

/* Allocation-free variant of sf37kv_decode(); no counterpart in the
 * reference.  For callers that cannot call cudaMalloc while decoding (an
 * engine whose memory pool owns the whole device, allocations frozen after
 * start-up, or a loop that cannot afford the device synchronization of a
 * first-use allocation): the split-K partials and counters live in a fixed
 * device array of SF37KV_NOALLOC_SCRATCH_BYTES compiled into the library,
 * which every GPU that loads the library holds until exit.  Same arguments
 * as sf37kv_decode() and the same kernels (the appended row is stored by the
 * attention kernel); the split plan may be coarser, so outputs agree with
 * sf37kv_decode() within the attention tolerance, not bit for bit, while the
 * appended cache rows are identical.  Limits: head_dim 128,
 * q_heads/kv_heads <= 16, at most 64 layers per call, layers x kv_heads <=
 * 4096; other sizes are rejected with SF37KV_EINVAL / SF37KV_EUNSUPPORTED
 * before anything is launched (the caches are left untouched).  The first
 * call on a device looks up the array's address (make it before any stream
 * capture).  All calls share the array: calls that overlap on the GPU race,
 * so serialize them. */
#define SF37KV_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u + 16384u)
int sf37kv_decode_noalloc(const sf37kv_decode_layer *layers, uint32_t n_layers,
                          uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                          int dtype, void *stream);

/* q/k head preparation fused into a decode step (the step before the
 * path: sf37_cuda_head_rms_norm_rope_qk_bf16_mapped, sf37_cuda.cu:2265-2316
 * and 6187-6240; CPU form sf37.c:2223-2231).  For each query head and each
 * head of the appended K row: RMS norm (double sum of squares,
 * scale = 1 / sqrtf(mean + eps)) times (w + 1) with bf16 weights w, then
 * split-half RoPE over the first rotary_dim dims at the layer's position:
 * pair (i, i + rotary_dim/2) rotated by (float)(pos * inv_freq(i)),
 * inv_freq(i) = theta^(-2i/rotary_dim), with the llama3 smoothing when
 * llama3 != 0 (sf37.c:1995-2013).  The reference model uses rotary_dim 64,
 * theta 5e6, llama3 on full layers and 128, 1e4, off on sliding layers
 * (sf37.c:1983-1993), eps 1e-5. */
typedef struct {
    const uint16_t *q_norm;  /* bf16 [head_dim], device */
    const uint16_t *k_norm;  /* bf16 [head_dim], device (needed with k_new) */
    double theta;
    uint32_t rotary_dim;     /* even, <= head_dim */
    uint32_t llama3;
    float eps;
    uint32_t reserved;
} sf37kv_qk_prep;

/* sf37kv_decode with layers[i].q and layers[i].k_new taken BEFORE head norm
 * and RoPE: prep[i] is applied inside the decode kernel, the cache receives
 * the prepared K row, and q/k_new in memory are left unchanged.  One launch
 * for all layers, as sf37kv_decode.  head_dim 128, group <= 16. */
int sf37kv_decode_prep(const sf37kv_decode_layer *layers, const sf37kv_qk_prep *prep,
                       uint32_t n_layers, uint32_t q_heads, uint32_t kv_heads,
                       uint32_t head_dim, int dtype, void *stream);

/* ---- the attention output projection (the step after the path) ----
 * out[r] = sum over 32-element blocks b of
 *   (float)dot(wq[r][b], xq[b]) * wscale[r][b] * xscale[b]
 * with Q8_0 weights (per row in_dim/32 blocks of 34 bytes: f16 scale, 32
 * int8) and x quantized to the same blocks (scale amax/127, codes
 * rint(x/scale) in [-128, 127]): sf37_q8_0_matvec (sf37_ops.c:57-123) and
 * sf37_cuda_matvec_q8_0 (sf37_cuda.cu:3319-3349, 3433-3461, 3708-3734).
 * x: f32 [in_dim] (e.g. the gated heads sf37kv_decode wrote), out: f32
 * [out_dim].  in_dim a multiple of 256; weights and x 16-byte aligned. */
typedef struct {
    const void *weights;
    const float *x;
    float *out;
} sf37kv_oproj_layer;

/* One launch for n_layers independent layers sharing in_dim / out_dim. */
int sf37kv_oproj_q8_0(const sf37kv_oproj_layer *layers, uint32_t n_layers, uint32_t in_dim,
                      uint32_t out_dim, void *stream);
/* The activation quantization alone: xq [n] int8, xscale [n/32] f32. */
int sf37kv_q8_0_quantize(const float *x, int8_t *xq, float *xscale, uint64_t n, void *stream);

/* Append n_tok rows per layer: row t -> slot (pos0 + t) % cap
 * (store_kv_cache_batch_kernel, sf37_cuda.cu:6355-6372). */
typedef struct {
    sf37kv_cache cache;
    uint32_t pos0;
    uint32_t n_tok;
    const float *k;        /* [n_tok][kv_dim] */
    const float *v;
} sf37kv_append_layer;
int sf37kv_append(const sf37kv_append_layer *layers, uint32_t n_layers,
                  uint32_t kv_dim, int dtype, void *stream);

/* Chunked prefill of one layer: the n_tok rows of the chunk must already be
 * appended; token t is a causal query at pos0 + t over rows
 * start_at(pos0+t) .. pos0+t (sf37_cuda.cu:3163-3317 semantics).
 * q: [n_tok][q_heads][head_dim] of q_type; gate: [n_tok][q_heads] f32 or
 * NULL; out: [n_tok][q_heads][head_dim] f32.  A sliding ring needs
 * cap >= window + n_tok (sf37.c:3083-3091) for exact results. */
int sf37kv_prefill(const sf37kv_cache *cache, const void *q, int q_type,
                   const float *gate, float *out, uint32_t pos0, uint32_t n_tok,
                   uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                   int dtype, void *stream);

/* ---- snapshot KV sections (bit-exact with the reference formats) ----
 * Byte size of one encoded row. */
uint64_t sf37kv_row_bytes(uint32_t kv_dim, int fmt, uint32_t group);

/* One layer of a snapshot pack/unpack: rows first_pos .. first_pos+rows-1
 * (ring slot % cap), written as K row then V row per position into
 * dst + offset (sf37.c:6980-7010, 7298-7320). */
typedef struct {
    sf37kv_cache cache;
    uint32_t first_pos;
    uint32_t rows;
    uint64_t offset;       /* byte offset of this layer's section in the buffer */
} sf37kv_pack_layer;

/* Gather/encode all layers into dst (device memory or device-mapped pinned
 * host memory).  variant: see sf37_cuda_kv_pack_rows_i8g. */
int sf37kv_pack(void *dst, const sf37kv_pack_layer *layers, uint32_t n_layers,
                uint32_t kv_dim, int dtype, int fmt, uint32_t group, int variant,
                void *stream);
/* Decode/scatter src back into the caches (the inverse of sf37kv_pack). */
int sf37kv_unpack(const void *src, const sf37kv_pack_layer *layers, uint32_t n_layers,
                  uint32_t kv_dim, int dtype, int fmt, uint32_t group, void *stream);

/* Pinned host memory for snapshot buffers (cudaHostAlloc, mapped). */
void *sf37kv_host_alloc(uint64_t bytes);
void sf37kv_host_free(void *p);

/* Whole snapshot KV section to host memory: packs on the device into a
 * staging buffer chunk by chunk and streams each chunk to host_dst with the
 * copy engine on a side stream, overlapping pack and copy.  Synchronous:
 * returns when host_dst holds the bytes.  host_dst should be pinned
 * (sf37kv_host_alloc) for full link speed. */
int sf37kv_pack_to_host(void *host_dst, const sf37kv_pack_layer *layers, uint32_t n_layers,
                        uint32_t kv_dim, int dtype, int fmt, uint32_t group, int variant);
int sf37kv_unpack_from_host(const void *host_src, const sf37kv_pack_layer *layers,
                            uint32_t n_layers, uint32_t kv_dim, int dtype, int fmt,
                            uint32_t group);

/* One GPU's KV-head slice of a multi-GPU record (sharded by KV head): the
 * caches hold elements [col0, col0 + kv_dim) of each full_kv_dim-element
 * row, and only those bytes of the full-width record rows are written
 * (read): raw, 4 kv_dim bytes at 4 col0 of each row; payload, the slice's
 * group scales and int8 codes in place (col0 and kv_dim multiples of
 * group; 64-element groups align with 128-element heads).  layers[i].offset
 * is the section's offset in the FULL layout.  Several GPUs can fill one
 * host buffer this way, each touching only its own columns.  Synchronous. */
int sf37kv_pack_slice_to_host(void *host_dst, const sf37kv_pack_layer *layers, uint32_t n_layers,
                              uint32_t kv_dim, uint32_t full_kv_dim, uint32_t col0, int dtype,
                              int fmt, uint32_t group, int variant);
int sf37kv_unpack_slice_from_host(const void *host_src, const sf37kv_pack_layer *layers,
                                  uint32_t n_layers, uint32_t kv_dim, uint32_t full_kv_dim,
                                  uint32_t col0, int dtype, int fmt, uint32_t group);

/* Synchronizes the device and returns the library's device error flag: 1
 * when a prefill kernel's bounded wait gave up, 2 when a multi-GPU gather or
 * reduce wait did (the kernel then stopped early and its output is
 * invalid), 0 otherwise, -1 if it cannot be read.  clear != 0 resets it. */
int sf37kv_device_error(int clear);

/* ---- multi-GPU output gather over peer memory (KV-head sharding) ----
 * Each rank allocates one device buffer (sf37kv_dev_alloc) holding the
 * gathered outputs [world][n_layers][q_heads_local][head_dim] f32, exports it
 * with sf37kv_ipc_handle and maps every other rank's with sf37kv_ipc_open.
 * peer_buf[p] / peer_flags[p]: rank p's buffer and its flag array (world
 * u32, zero-initialized) as mapped in this process; my_flags = this rank's
 * flag array; done_counter: one zeroed device u32 of this rank. */
typedef struct {
    void *peer_buf[8];
    void *peer_flags[8];
    void *my_flags;
    void *done_counter;
    uint32_t world;
    uint32_t rank;
} sf37kv_peer_gather;

/* Zero-filled device memory (cudaMalloc; freed with sf37kv_dev_free). */
void *sf37kv_dev_alloc(uint64_t bytes);
void sf37kv_dev_free(void *p);
/* CUDA IPC of a whole sf37kv_dev_alloc allocation; handle_out: 64 bytes. */
int sf37kv_ipc_handle(void *dev_ptr, void *handle_out);
void *sf37kv_ipc_open(const void *handle);
void sf37kv_ipc_close(void *p);

/* sf37kv_decode on this rank's KV-head slice (1..64 layers), with every
 * output head stored into all ranks' gather buffers, laid out as f32
 * [2][world][n_layers][q_heads][head_dim] with half (epoch & 1); layers[i].out
 * is ignored (the output lands in this rank's own buffer at
 * [epoch & 1][rank][i]).  This rank's epoch flag is raised in every rank's
 * flag array after its last output is stored.  Epochs must increase by one
 * per step, starting at 1 with zeroed flags.  Multi-GPU form of
 * sf37_cuda_attention_decode_heads (sf37_cuda.h:108-118); the reference runs
 * on one GPU and has no counterpart for the gather itself. */
int sf37kv_decode_gather(const sf37kv_decode_layer *layers, uint32_t n_layers,
                         uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                         int dtype, const sf37kv_peer_gather *g, uint32_t epoch,
                         void *stream);
/* Waits on the stream (bounded, about 2 s) until every rank raised `epoch`;
 * on timeout the device error flag is set to 2 (sf37kv_device_error). */
int sf37kv_gather_wait(const sf37kv_peer_gather *g, uint32_t epoch, void *stream);

/* Row-parallel o_proj across the KV-head shards: rank r passes its query
 * heads' slice of x (in_dim = 8192/N elements) and the matching column
 * slice of every weight row (weights = row start + r * in_dim/32 * 34
 * bytes, row_stride = the full row's bytes).  Each rank's partial rows are
 * stored into every rank's buffer of g (f32 [2][world][n_layers][out_dim],
 * half epoch & 1, slot rank; layers[i].out is ignored) and its epoch flag
 * is raised after the last store; sf37kv_oproj_reduce then waits (bounded,
 * about 2 s; error flag 2 on timeout) and sums the slots in rank order into
 * out [n_layers][out_dim] (the same bits on every rank).  1..64 layers. */
int sf37kv_oproj_q8_0_shard(const sf37kv_oproj_layer *layers, uint32_t n_layers, uint32_t in_dim,
                            uint32_t out_dim, uint64_t row_stride, const sf37kv_peer_gather *g,
                            uint32_t epoch, void *stream);
int sf37kv_oproj_reduce(const sf37kv_peer_gather *g, uint32_t n_layers, uint32_t out_dim,
                        uint32_t epoch, float *out, void *stream);

/* Number of kernel launches this library has issued (process total). */
uint64_t sf37kv_launch_count(void);

/* ---- Decode cache sizing (the reference engine's rules) ----
 * sf37kv_sliding_cache_cap: ring rows of a sliding-window layer for a context
 * of ctx_size and a prefill chunk of prefill_cap: align256(512 + chunk),
 * clamped to [window, min(ctx_size, 8192)] (cuda_sliding_cache_cap,
 * sf37.c:3067-3081).  sf37kv_sliding_prefill_cap: the largest chunk such a
 * ring prefills exactly, cache_cap - window (cuda_sliding_cache_prefill_cap,
 * sf37.c:3083-3091).  sf37kv_kv_cache_bytes: K+V bytes of one layer's cache
 * (cuda_decode_kv_bytes_for_cap, sf37.c:3093-3096, for dtype f32; f16 caches
 * take half).  sf37kv_prefill_default_chunk: the chunk the engine picks from
 * the device's free memory (4096 / 2048 / 1024 / 512 at 24 / 12 / 6 GiB,
 * cuda_prefill_default_chunk, sf37.c:5131-5140; its environment override is
 * the caller's).  sf37kv_plan_caches: every layer's cap as
 * cuda_decode_state_init lays them out (sf37.c:3189-3211: layers il % 4 == 0
 * hold the whole context, the others a sliding ring). */
#define SF37KV_PLAN_MAX_LAYERS 64
typedef struct {
    uint32_t ctx_size;       /* clamped to [1, 262144] */
    uint32_t window;         /* sliding window, min(512, ctx_size) */
    uint32_t sliding_cap;    /* ring rows of every sliding layer */
    uint32_t prefill_cap;    /* largest exact prefill chunk */
    uint32_t full_layers, sliding_layers;
    uint32_t cap[SF37KV_PLAN_MAX_LAYERS];
    uint32_t sliding[SF37KV_PLAN_MAX_LAYERS];
    uint64_t kv_cache_bytes; /* all layers, K and V, of the given dtype */
} sf37kv_cache_plan;
uint32_t sf37kv_sliding_cache_cap(uint32_t ctx_size, uint32_t prefill_cap);
uint32_t sf37kv_sliding_prefill_cap(uint32_t ctx_size, uint32_t cache_cap);
uint64_t sf37kv_kv_cache_bytes(uint32_t cap, uint32_t kv_heads, uint32_t head_dim, int dtype);
uint32_t sf37kv_prefill_default_chunk(uint64_t free_bytes);
int sf37kv_plan_caches(uint32_t ctx_size, uint32_t prefill_chunk, uint32_t n_layers, uint32_t kv_heads,
                       uint32_t head_dim, int dtype, sf37kv_cache_plan *plan);
/* The managed-KV-cache policy of sf37_cuda_should_use_managed_kv_cache
 * (sf37_cuda.cu:1766-1800) on given free/total device bytes instead of a
 * live cudaMemGetInfo: 1 = allocate the KV cache as managed memory. */
int sf37kv_managed_kv_policy(uint64_t kv_cache_bytes, uint64_t context_bytes, uint64_t free_bytes,
                             uint64_t total_bytes);

#ifdef __cplusplus
}
#endif

#endif
