/*
 * Session KV checkpoints of libsf37kv: the raw snapshot (format 2) and the
 * int8-grouped payload (format 3) that sf37_kvstore stores, written from and
 * restored into device KV caches with the bulk pack kernels.
 *
 * Same bytes as the reference's CUDA-backend session code:
 *   sf37kv_session_snapshot_bytes  <- sf37_session_snapshot_bytes  (sf37.c:6809-6820)
 *   sf37kv_session_payload_bytes   <- sf37_session_payload_bytes   (sf37.c:6822-6835)
 *   sf37kv_session_save_snapshot   <- sf37_session_save_snapshot   (sf37.c:7235-7345)
 *   sf37kv_session_load_snapshot   <- sf37_session_load_snapshot   (sf37.c:7347-7500)
 *   sf37kv_session_save_payload    <- sf37_session_save_payload    (sf37.c:6922-7036)
 *   sf37kv_session_load_payload    <- sf37_session_load_payload    (sf37.c:7038-7233)
 * The reference declares these in sf37.h:153-164 with an sf37_session that
 * needs a loaded model; here the session state the formats carry is passed
 * explicitly (sf37kv_session).  Return codes follow sf37.h: 0 = success,
 * nonzero = failure with a message in err (and in sf37kv_last_error()); the
 * messages are the reference's.
 *
 * Differences, all below the format: the KV rows move as one device pack per
 * layer chunk plus one large copy instead of two 4 KiB cudaMemcpy per row,
 * and the payload streams straight between pinned buffers and the file
 * descriptor (no staging file).
 */
#ifndef SF37KV_SESSION_H
#define SF37KV_SESSION_H

#include <stddef.h>
#include <stdint.h>

#include "sf37kv.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Model dimensions the formats record (header words 5-9) and the row rules
 * the loaders check.  sf37kv_session_layout_default() gives the reference
 * model's: 45 layers, 8 KV heads, head_dim 128, vocab 128896, embd 4096,
 * sliding window 512, full-attention layers il % 4 == 0, payload group 64
 * (sf37.c:32-70, 1983-1985). */
typedef struct {
    uint32_t n_layers;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t vocab;
    uint32_t embd;
    uint32_t sliding_window;
    uint32_t full_every;     /* layer il is full attention iff il % full_every == 0 */
    uint32_t payload_group;  /* int8 group size of the payload rows */
} sf37kv_session_layout;

sf37kv_session_layout sf37kv_session_layout_default(void);

/* The session state a checkpoint holds.  tokens, logits and hidden are host
 * memory; caches[il] are the device caches of layer il (dtype SF37KV_F32,
 * the reference's, or SF37KV_F16).  Logical position p of layer il lives in
 * slot p % caches[il].cap.  Layer il holds min(min(n_tokens, ctx_size),
 * caches[il].cap) live rows, the last positions before n_tokens
 * (sf37.c:6495-6528).  The loaders write tokens (capacity ctx_size), logits,
 * hidden and n_tokens. */
typedef struct {
    sf37kv_session_layout layout;
    int32_t ctx_size;
    uint32_t n_tokens;
    int32_t *tokens;
    float *logits;
    float *hidden;
    const sf37kv_cache *caches;
    int dtype;
    uint32_t backend_kind;  /* header word 10: 1 = CUDA (the KV row order written here) */
} sf37kv_session;

uint64_t sf37kv_session_snapshot_bytes(const sf37kv_session *s);
uint64_t sf37kv_session_payload_bytes(const sf37kv_session *s);

/* Raw snapshot into dst (host memory; pinned via sf37kv_host_alloc for full
 * link speed).  *len receives the bytes written.  Fails if dst_cap is short. */
int sf37kv_session_save_snapshot(const sf37kv_session *s, void *dst, uint64_t dst_cap,
                                 uint64_t *len, char *err, size_t errlen);
/* Restores a raw snapshot: validates it against s (ctx, layout, row counts,
 * caps) like the reference, then writes the caches' live slots and the host
 * fields.  On failure the caches may be partly written (as the reference). */
int sf37kv_session_load_snapshot(sf37kv_session *s, const void *src, uint64_t len,
                                 char *err, size_t errlen);

/* Payload to / from a file descriptor at its current offset.  The loader
 * reads exactly payload_bytes (the stored record size). */
int sf37kv_session_save_payload(const sf37kv_session *s, int fd, char *err, size_t errlen);
int sf37kv_session_load_payload(sf37kv_session *s, int fd, uint64_t payload_bytes, char *err,
                                size_t errlen);

#ifdef __cplusplus
}
#endif

#endif
