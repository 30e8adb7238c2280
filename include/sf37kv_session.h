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

/* ---- sf37_kvstore records (the files the server's disk KV cache holds) ----
 * Record = 48-byte header, 4-byte little-endian text length, the cached
 * text, then the session payload (format 3) and an optional trailer owned
 * by the server's hooks.  The file is named "<sha1 of text>.kv".
 *   sf37kv_kvstore_fill_header  <- sf37_kvstore_fill_header (sf37_kvstore.c:399-421)
 *   sf37kv_kvstore_parse_header <- sf37_kvstore_read_header (sf37_kvstore.c:423-446):
 *                                  1 when magic/version/ABI match, tokens != 0
 *                                  and quant_bits == 3; h holds the header
 *                                  and the text length (52 bytes)
 *   sf37kv_sha1_hex             <- sf37_kvstore_sha1_bytes_hex (sf37_kvstore.c:327)
 *   sf37kv_kvstore_save         <- the record write of sf37_kvstore_store_live_prefix_text
 *                                  (sf37_kvstore.c:1052-1079), without the trailer:
 *                                  writes at fd's current offset; the payload
 *                                  streams from the device caches (no staging
 *                                  file); model 37, quant 3, hits 0, created =
 *                                  last used = now
 *   sf37kv_kvstore_load         <- the checks and payload load of
 *                                  sf37_kvstore_try_load_text (sf37_kvstore.c:1249-1303),
 *                                  reading from fd's current offset; prompt is
 *                                  the incoming prompt text, sha_expected the
 *                                  file's name key or NULL.  Messages are the
 *                                  reference's ("invalid header", "cached text
 *                                  hash mismatch", ...). */
#define SF37KV_KVSTORE_HEADER 48
#define SF37KV_KVSTORE_MODEL_ID 37
#define SF37KV_KVSTORE_QUANT_BITS 3
#define SF37KV_KVSTORE_REASON_MAX 6
typedef struct {
    uint8_t quant_bits, model_id, reason, ext_flags;
    uint32_t tokens, hits, ctx_size, text_bytes;
    uint64_t created_at, last_used, payload_bytes;
} sf37kv_kvstore_entry;
void sf37kv_kvstore_fill_header(uint8_t h[SF37KV_KVSTORE_HEADER], uint8_t model_id, uint8_t quant_bits,
                                uint8_t reason, uint8_t ext_flags, uint32_t tokens, uint32_t hits,
                                uint32_t ctx_size, uint64_t created_at, uint64_t last_used,
                                uint64_t payload_bytes);
int sf37kv_kvstore_parse_header(const uint8_t h[SF37KV_KVSTORE_HEADER + 4], sf37kv_kvstore_entry *e);
void sf37kv_sha1_hex(const void *data, size_t len, char out[41]);
int sf37kv_kvstore_save(const sf37kv_session *s, int fd, const char *text, uint32_t text_len, uint8_t reason,
                        uint8_t ext_flags, uint64_t now, uint64_t *record_bytes, char *err, size_t errlen);
int sf37kv_kvstore_load(sf37kv_session *s, int fd, const char *prompt, size_t prompt_len,
                        const char *sha_expected, uint32_t *tokens_loaded, char *err, size_t errlen);

#ifdef __cplusplus
}
#endif

#endif
