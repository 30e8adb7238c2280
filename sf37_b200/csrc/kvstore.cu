// sf37_kvstore records written from / restored into device KV caches.
//
// A kvstore file (sf37_kvstore.c) is: a 48-byte header
// (sf37_kvstore_fill_header, sf37_kvstore.c:399-421), the 4-byte
// little-endian length of the cached text, the text, then the session's
// int8-grouped payload (format 3) and an optional trailer that the server's
// hooks own.  The file is named by the SHA-1 of the text
// (sf37_kvstore_path_for_sha, sf37_kvstore.c:354-359).  The reference store
// path (sf37_kvstore_store_live_prefix_text, sf37_kvstore.c:929-1158) first
// stages the whole payload through a temporary file and then copies it into
// the record; here the payload streams from the device caches straight into
// the record's file descriptor (sf37kv_session_save_payload), and the load
// path (sf37_kvstore_try_load_text, sf37_kvstore.c:1218-1357) streams it back
// with the same checks and messages.
//
// Host code only.
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <unistd.h>

#include "kv_internal.cuh"
#include "../../include/sf37kv_session.h"

namespace {

// Header constants (sf37_kvstore.c:28-37).
constexpr uint8_t kMagic[3] = {'K', 'V', 'C'};
constexpr uint8_t kVersion = 1;
constexpr uint8_t kPayloadAbi = 2;

void put32(uint8_t *p, uint32_t v) {
    for (int i = 0; i < 4; i++) p[i] = (uint8_t)(v >> (8 * i));
}
void put64(uint8_t *p, uint64_t v) {
    for (int i = 0; i < 8; i++) p[i] = (uint8_t)(v >> (8 * i));
}
uint32_t get32(const uint8_t *p) {
    uint32_t v = 0;
    for (int i = 3; i >= 0; i--) v = (v << 8) | p[i];
    return v;
}
uint64_t get64(const uint8_t *p) {
    uint64_t v = 0;
    for (int i = 7; i >= 0; i--) v = (v << 8) | p[i];
    return v;
}

// SHA-1 (FIPS 180-4): 512-bit blocks, 80 rounds, big-endian length pad.
struct Sha1 {
    uint32_t h[5] = {0x67452301u, 0xEFCDAB89u, 0x98BADCFEu, 0x10325476u, 0xC3D2E1F0u};
    uint8_t buf[64];
    uint64_t bits = 0;
    uint32_t fill = 0;

    static uint32_t rol(uint32_t x, int s) { return (x << s) | (x >> (32 - s)); }
    void block(const uint8_t *b) {
        uint32_t w[80];
        for (int i = 0; i < 16; i++)
            w[i] = ((uint32_t)b[4 * i] << 24) | ((uint32_t)b[4 * i + 1] << 16) | ((uint32_t)b[4 * i + 2] << 8) |
                   (uint32_t)b[4 * i + 3];
        for (int i = 16; i < 80; i++) w[i] = rol(w[i - 3] ^ w[i - 8] ^ w[i - 14] ^ w[i - 16], 1);
        uint32_t a = h[0], bb = h[1], c = h[2], d = h[3], e = h[4];
        for (int i = 0; i < 80; i++) {
            uint32_t f, k;
            if (i < 20) {
                f = (bb & c) | (~bb & d);
                k = 0x5A827999u;
            } else if (i < 40) {
                f = bb ^ c ^ d;
                k = 0x6ED9EBA1u;
            } else if (i < 60) {
                f = (bb & c) | (bb & d) | (c & d);
                k = 0x8F1BBCDCu;
            } else {
                f = bb ^ c ^ d;
                k = 0xCA62C1D6u;
            }
            const uint32_t t = rol(a, 5) + f + e + k + w[i];
            e = d;
            d = c;
            c = rol(bb, 30);
            bb = a;
            a = t;
        }
        h[0] += a;
        h[1] += bb;
        h[2] += c;
        h[3] += d;
        h[4] += e;
    }
    void update(const uint8_t *p, size_t n) {
        bits += (uint64_t)n * 8u;
        while (n) {
            const uint32_t take = (uint32_t)std::min<size_t>(n, 64u - fill);
            memcpy(buf + fill, p, take);
            fill += take;
            p += take;
            n -= take;
            if (fill == 64) {
                block(buf);
                fill = 0;
            }
        }
    }
    void final(uint8_t out[20]) {
        const uint64_t total = bits;
        const uint8_t one = 0x80, zero = 0;
        update(&one, 1);
        while (fill != 56) update(&zero, 1);
        uint8_t len[8];
        for (int i = 0; i < 8; i++) len[i] = (uint8_t)(total >> (56 - 8 * i));
        update(len, 8);
        for (int i = 0; i < 5; i++)
            for (int j = 0; j < 4; j++) out[4 * i + j] = (uint8_t)(h[i] >> (24 - 8 * j));
    }
};

int fail(char *err, size_t errlen, int code, const char *msg) {
    if (err && errlen) snprintf(err, errlen, "%s", msg);
    return sf37kv::set_error(code, "%s", msg);
}

bool write_all(int fd, const void *p, size_t n) {
    const uint8_t *b = static_cast<const uint8_t *>(p);
    while (n) {
        const ssize_t w = write(fd, b, n);
        if (w < 0 && errno == EINTR) continue;
        if (w <= 0) return false;
        b += w;
        n -= (size_t)w;
    }
    return true;
}

bool read_all(int fd, void *p, size_t n) {
    uint8_t *b = static_cast<uint8_t *>(p);
    while (n) {
        const ssize_t r = read(fd, b, n);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        b += r;
        n -= (size_t)r;
    }
    return true;
}

}  // namespace

extern "C" void sf37kv_sha1_hex(const void *data, size_t len, char out[41]) {
    Sha1 s;
    s.update(static_cast<const uint8_t *>(data), len);
    uint8_t d[20];
    s.final(d);
    static const char hex[] = "0123456789abcdef";
    for (int i = 0; i < 20; i++) {
        out[2 * i] = hex[d[i] >> 4];
        out[2 * i + 1] = hex[d[i] & 15];
    }
    out[40] = '\0';
}

extern "C" void sf37kv_kvstore_fill_header(uint8_t h[SF37KV_KVSTORE_HEADER], uint8_t model_id, uint8_t quant_bits,
                                           uint8_t reason, uint8_t ext_flags, uint32_t tokens, uint32_t hits,
                                           uint32_t ctx_size, uint64_t created_at, uint64_t last_used,
                                           uint64_t payload_bytes) {
    memset(h, 0, SF37KV_KVSTORE_HEADER);
    h[0] = kMagic[0];
    h[1] = kMagic[1];
    h[2] = kMagic[2];
    h[3] = kVersion;
    h[4] = quant_bits;
    h[5] = reason;
    h[6] = ext_flags;
    h[7] = model_id;
    put32(h + 8, tokens);
    put32(h + 12, hits);
    put32(h + 16, ctx_size);
    h[20] = kPayloadAbi;
    put64(h + 24, created_at);
    put64(h + 32, last_used);
    put64(h + 40, payload_bytes);
}

extern "C" int sf37kv_kvstore_parse_header(const uint8_t h[SF37KV_KVSTORE_HEADER + 4], sf37kv_kvstore_entry *e) {
    if (!h || !e) return 0;
    if (h[0] != kMagic[0] || h[1] != kMagic[1] || h[2] != kMagic[2] || h[3] != kVersion) return 0;
    if (h[20] != kPayloadAbi) return 0;
    memset(e, 0, sizeof(*e));
    e->quant_bits = h[4];
    e->reason = h[5] <= SF37KV_KVSTORE_REASON_MAX ? h[5] : 0;
    e->ext_flags = h[6];
    e->model_id = h[7];
    e->tokens = get32(h + 8);
    e->hits = get32(h + 12);
    e->ctx_size = get32(h + 16);
    e->created_at = get64(h + 24);
    e->last_used = get64(h + 32);
    e->payload_bytes = get64(h + 40);
    e->text_bytes = get32(h + SF37KV_KVSTORE_HEADER);
    return e->tokens != 0 && e->quant_bits == SF37KV_KVSTORE_QUANT_BITS;
}

extern "C" int sf37kv_kvstore_save(const sf37kv_session *s, int fd, const char *text, uint32_t text_len,
                                   uint8_t reason, uint8_t ext_flags, uint64_t now, uint64_t *record_bytes,
                                   char *err, size_t errlen) {
    if (!s || fd < 0 || (!text && text_len)) return fail(err, errlen, SF37KV_EINVAL, "kvstore save: bad arguments");
    if (s->n_tokens == 0) return fail(err, errlen, SF37KV_EINVAL, "kvstore save: session holds no tokens");
    const uint64_t payload = sf37kv_session_payload_bytes(s);
    uint8_t h[SF37KV_KVSTORE_HEADER + 4];
    sf37kv_kvstore_fill_header(h, SF37KV_KVSTORE_MODEL_ID, SF37KV_KVSTORE_QUANT_BITS, reason, ext_flags, s->n_tokens,
                               0, (uint32_t)s->ctx_size, now, now, payload);
    put32(h + SF37KV_KVSTORE_HEADER, text_len);
    if (!write_all(fd, h, sizeof(h)) || !write_all(fd, text, text_len))
        return fail(err, errlen, SF37KV_ECUDA, strerror(errno ? errno : EIO));
    if (int rc = sf37kv_session_save_payload(s, fd, err, errlen)) return rc;
    if (record_bytes) *record_bytes = sizeof(h) + (uint64_t)text_len + payload;
    return SF37KV_OK;
}

extern "C" int sf37kv_kvstore_load(sf37kv_session *s, int fd, const char *prompt, size_t prompt_len,
                                   const char *sha_expected, uint32_t *tokens_loaded, char *err, size_t errlen) {
    if (tokens_loaded) *tokens_loaded = 0;
    if (!s || fd < 0 || (!prompt && prompt_len)) return fail(err, errlen, SF37KV_EINVAL, "kvstore load: bad arguments");
    uint8_t h[SF37KV_KVSTORE_HEADER + 4];
    sf37kv_kvstore_entry e;
    if (!read_all(fd, h, sizeof(h)) || !sf37kv_kvstore_parse_header(h, &e))
        return fail(err, errlen, SF37KV_EINVAL, "invalid header");
    if (e.model_id != SF37KV_KVSTORE_MODEL_ID)
        return fail(err, errlen, SF37KV_EINVAL, "cached checkpoint was written for a different model");
    if ((uint64_t)e.text_bytes > prompt_len) return fail(err, errlen, SF37KV_EINVAL, "cached text is longer than prompt");
    char *text = static_cast<char *>(malloc((size_t)e.text_bytes + 1u));
    if (!text) return fail(err, errlen, SF37KV_ENOMEM, "kvstore load: out of host memory");
    int rc = SF37KV_OK;
    if (!read_all(fd, text, e.text_bytes)) {
        rc = fail(err, errlen, SF37KV_EINVAL, "truncated cached text");
    } else {
        char sha[41];
        sf37kv_sha1_hex(text, e.text_bytes, sha);
        if (sha_expected && strncmp(sha, sha_expected, 40) != 0)
            rc = fail(err, errlen, SF37KV_EINVAL, "cached text hash mismatch");
        else if (e.text_bytes && memcmp(prompt, text, e.text_bytes) != 0)
            rc = fail(err, errlen, SF37KV_EINVAL, "cached text prefix mismatch");
    }
    free(text);
    if (rc) return rc;
    if ((rc = sf37kv_session_load_payload(s, fd, e.payload_bytes, err, errlen))) return rc;
    if (s->n_tokens != e.tokens) {
        s->n_tokens = 0;  // the reference rewinds the session and discards the file
        return fail(err, errlen, SF37KV_EINVAL, "kv cache discarded corrupt text-prefix payload");
    }
    if (tokens_loaded) *tokens_loaded = e.tokens;
    return SF37KV_OK;
}
