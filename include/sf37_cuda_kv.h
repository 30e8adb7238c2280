/*
 * Drop-in C ABI for the SF37 KV-cache hot path.
 *
 * These are the reference's own entry points from sf37_cuda.h, with the same
 * names, argument meaning, fp32 cache element type and return convention
 * (int 1 = success, 0 = failure, with a message on stderr).  A build of the
 * reference engine (sf37.c, sf37_server.c) that links libsf37kv.so in place of
 * the reference's sf37_cuda.o for these symbols gets the B200 kernels with no
 * source change.  Each declaration names the reference declaration it
 * replaces (file:line in the reference tree).
 *
 * Conventions kept from the reference:
 *   - every tensor is an opaque handle whose first two members are
 *     {void *ptr; uint64_t bytes;}; callers may build views by value
 *     (sf37_cuda.cu:32-35, sf37.c builds such views);
 *   - argument sizes are validated against tensor byte sizes before launch;
 *   - launches are asynchronous on the library stream (the legacy default
 *     stream unless sf37kv_set_stream() chose another); tensor read/write are
 *     synchronous;
 *   - not thread-safe: the library keeps one process-wide split-K scratch.
 */
#ifndef SF37_CUDA_KV_H
#define SF37_CUDA_KV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct sf37_cuda_tensor sf37_cuda_tensor;
struct sf37_cuda_tensor {
    void *ptr;
    uint64_t bytes;
};

/* sf37_cuda.h:12-19 */
int sf37_cuda_device_count(void);
int sf37_cuda_init(void);
void sf37_cuda_cleanup(void);
int sf37_cuda_synchronize(void);
int sf37_cuda_memory_info(uint64_t *free_bytes, uint64_t *total_bytes);

/* Tensor API, sf37_cuda.h:39-50 */
sf37_cuda_tensor *sf37_cuda_tensor_alloc(uint64_t bytes);
sf37_cuda_tensor *sf37_cuda_tensor_alloc_managed(uint64_t bytes);
void sf37_cuda_tensor_free(sf37_cuda_tensor *tensor);
uint64_t sf37_cuda_tensor_bytes(const sf37_cuda_tensor *tensor);
int sf37_cuda_tensor_write(sf37_cuda_tensor *tensor, uint64_t offset,
                           const void *data, uint64_t bytes);
int sf37_cuda_tensor_read(const sf37_cuda_tensor *tensor, uint64_t offset,
                          void *data, uint64_t bytes);
int sf37_cuda_tensor_copy(sf37_cuda_tensor *dst, uint64_t dst_offset,
                          const sf37_cuda_tensor *src, uint64_t src_offset,
                          uint64_t bytes);
int sf37_cuda_tensor_fill_f32(sf37_cuda_tensor *tensor, float value, uint64_t count);

/* sf37_cuda.h:102-107: position-0 shortcut, out = v[kvh] * sigmoid(gate). */
int sf37_cuda_gqa_single_token_heads(sf37_cuda_tensor *out_heads,
                                     const sf37_cuda_tensor *v,
                                     const sf37_cuda_tensor *head_gate,
                                     uint32_t q_heads,
                                     uint32_t kv_heads,
                                     uint32_t head_dim);

/* sf37_cuda.h:108-119: decode over logical rows 0..n_cache-1 (sliding keeps
 * the last `window`), ring slot r % cache_cap, requires n_cache <= cache_cap. */
int sf37_cuda_attention_decode_heads(sf37_cuda_tensor *out_heads,
                                     const sf37_cuda_tensor *q,
                                     const sf37_cuda_tensor *k_cache,
                                     const sf37_cuda_tensor *v_cache,
                                     const sf37_cuda_tensor *head_gate,
                                     uint32_t n_cache,
                                     uint32_t cache_cap,
                                     uint32_t q_heads,
                                     uint32_t kv_heads,
                                     uint32_t head_dim,
                                     int sliding,
                                     uint32_t window);

/* sf37_cuda.h:120-131: decode of the query at position pos; rows
 * max(pos+1-cap, pos+1-window if sliding, 0) .. pos, ring slot r % cap. */
int sf37_cuda_attention_decode_heads_at(sf37_cuda_tensor *out_heads,
                                        const sf37_cuda_tensor *q,
                                        const sf37_cuda_tensor *k_cache,
                                        const sf37_cuda_tensor *v_cache,
                                        const sf37_cuda_tensor *head_gate,
                                        uint32_t pos,
                                        uint32_t cache_cap,
                                        uint32_t q_heads,
                                        uint32_t kv_heads,
                                        uint32_t head_dim,
                                        int sliding,
                                        uint32_t window);

/* sf37_cuda.h:132-133 (policy restated, sf37_cuda.cu:1766-1800). */
int sf37_cuda_should_use_managed_kv_cache(uint64_t kv_cache_bytes,
                                          uint64_t context_bytes);

/* sf37_cuda.h:134-137: Q8_0 matvec (the attention output projection after
 * the decode; sf37_cuda.cu:3708-3734).  out f32 [out_dim], weights
 * out_dim x (in_dim/32) blocks of 34 bytes, x f32 [in_dim].  Same sizes
 * checks and 1/0 return; this build needs in_dim % 256 == 0 (true for every
 * SF37 projection) and returns 0 with a message otherwise. */
int sf37_cuda_matvec_q8_0(sf37_cuda_tensor *out,
                          const sf37_cuda_tensor *weights,
                          uint64_t in_dim, uint64_t out_dim,
                          const sf37_cuda_tensor *x);

/* sf37_cuda.h:241-248: append n_tok rows into ring slots (pos0+t) % cap. */
int sf37_cuda_store_kv_cache_batch(sf37_cuda_tensor *k_cache,
                                   sf37_cuda_tensor *v_cache,
                                   const sf37_cuda_tensor *k,
                                   const sf37_cuda_tensor *v,
                                   uint32_t pos0,
                                   uint32_t n_tok,
                                   uint32_t cache_cap,
                                   uint32_t kv_dim);

/* sf37_cuda.h:249-261: causal chunk attention, token t at pos0+t. */
int sf37_cuda_attention_prefill_heads(sf37_cuda_tensor *out_heads,
                                      const sf37_cuda_tensor *q,
                                      const sf37_cuda_tensor *k_cache,
                                      const sf37_cuda_tensor *v_cache,
                                      const sf37_cuda_tensor *head_gate,
                                      uint32_t pos0,
                                      uint32_t n_tok,
                                      uint32_t cache_cap,
                                      uint32_t q_heads,
                                      uint32_t kv_heads,
                                      uint32_t head_dim,
                                      int sliding,
                                      uint32_t window);

/*
 * Bulk snapshot KV export/import in the reference's style (int 1/0, tensor
 * handles).  They replace the per-row loops of the CUDA backend in
 * sf37_session_save_snapshot (sf37.c:7298-7320), sf37_session_load_snapshot
 * (sf37.c:7410-7432), sf37_session_save_payload (sf37.c:6980-7010) and
 * sf37_session_load_payload (sf37.c:7146-7185), producing the same bytes:
 * for r in 0..rows-1 at ring slot (first_pos + r) % cache_cap, the K row then
 * the V row.  host_dst/host_src is ordinary or pinned host memory of
 * rows * 2 * row_bytes, row_bytes = kv_dim*4 (raw) or
 * ceil(kv_dim/group)*4 + kv_dim (int8-grouped).  They return after the
 * copy has completed.
 */
int sf37_cuda_kv_pack_rows_f32(void *host_dst,
                               const sf37_cuda_tensor *k_cache,
                               const sf37_cuda_tensor *v_cache,
                               uint32_t first_pos, uint32_t rows,
                               uint32_t cache_cap, uint32_t kv_dim);
int sf37_cuda_kv_unpack_rows_f32(const void *host_src,
                                 sf37_cuda_tensor *k_cache,
                                 sf37_cuda_tensor *v_cache,
                                 uint32_t first_pos, uint32_t rows,
                                 uint32_t cache_cap, uint32_t kv_dim);
/* variant: 1 = the bytes of the reference built with its Makefile flags
 * (-ffast-math: scale = max*(1/127), q = rint(x * (1/scale))); 0 = the
 * source-literal IEEE arithmetic (scale = max/127, q = rint(x / scale)). */
int sf37_cuda_kv_pack_rows_i8g(void *host_dst,
                               const sf37_cuda_tensor *k_cache,
                               const sf37_cuda_tensor *v_cache,
                               uint32_t first_pos, uint32_t rows,
                               uint32_t cache_cap, uint32_t kv_dim,
                               uint32_t group, int variant);
int sf37_cuda_kv_unpack_rows_i8g(const void *host_src,
                                 sf37_cuda_tensor *k_cache,
                                 sf37_cuda_tensor *v_cache,
                                 uint32_t first_pos, uint32_t rows,
                                 uint32_t cache_cap, uint32_t kv_dim,
                                 uint32_t group);

#ifdef __cplusplus
}
#endif

#endif
