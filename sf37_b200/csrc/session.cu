// Session KV checkpoints: the raw snapshot (format 2) and the int8-grouped
// payload (format 3) of sf37.c, written from and restored into device caches.
//
// Format (both little-endian, as the reference writes them with fwrite /
// memcpy on x86):
//   u32 header[11] (snapshot)  {magic 0x37334653, 2, ctx, tokens, live_rows,
//                               layers, kv_heads, head_dim, vocab, embd, backend}
//   u32 header[15] (payload)   {magic 0x37375053, 3, ..., backend,
//                               kv_enc 1, group, groups, encoded_row_bytes}
//   u32 row_counts[layers]; u32 tokens[tokens]; f32 logits[vocab];
//   f32 hidden[embd]; then per layer, per live row: the K row then the V row
//   (raw f32, or the payload row encoding).
// sf37.c:7262-7320 (snapshot writer), 6934-7010 (payload writer),
// 7347-7478 and 7038-7185 (the loaders and their checks, restated in order
// with the same messages).
#include <cerrno>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <thread>
#include <unistd.h>
#include <vector>

#include "kv_internal.cuh"
#include "../../include/sf37kv_session.h"

namespace sf37kv {
namespace {

constexpr uint32_t kSnapMagic = 0x37334653u, kSnapVersion = 2u, kSnapFields = 11u;
constexpr uint32_t kPayMagic = 0x37375053u, kPayVersion = 3u, kPayFields = 15u;
constexpr uint32_t kKvI8Grouped = 1u;
constexpr uint64_t kIoChunk = 8ull << 20;

// Formats the message into err (the reference's snapshot_set_err) and into
// the library's last error; returns 1 (the reference's failure code).
int fail(char *err, size_t errlen, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (err && errlen) snprintf(err, errlen, "%s", buf);
    set_error(SF37KV_EINVAL, "%s", buf);
    return 1;
}

// Library-level failure (CUDA, bad descriptor): keeps sf37kv_last_error's
// message and copies it into err.
int fail_last(char *err, size_t errlen, const char *what) {
    const char *m = sf37kv_last_error();
    char buf[600];
    snprintf(buf, sizeof(buf), "%s: %s", what, m ? m : "");
    if (err && errlen) snprintf(err, errlen, "%s", buf);
    set_error(SF37KV_EINVAL, "%s", buf);
    return 1;
}

uint32_t kv_row(const sf37kv_session_layout &L) { return L.kv_heads * L.head_dim; }
uint32_t groups_per_row(uint32_t elems, uint32_t group) { return group ? (elems + group - 1u) / group : 0; }
uint64_t encoded_row_bytes(uint32_t elems, uint32_t group) {
    return (uint64_t)groups_per_row(elems, group) * 4u + elems;
}
bool layer_full(const sf37kv_session_layout &L, uint32_t il) { return L.full_every && il % L.full_every == 0; }

// session_live_kv_rows / session_layer_live_kv_rows (sf37.c:6495-6521) for
// a CUDA session: min(tokens, ctx), clamped by each layer's cache cap.
uint32_t live_rows(const sf37kv_session *s) {
    if (s->n_tokens == 0 || s->ctx_size <= 0) return 0;
    return s->n_tokens < (uint32_t)s->ctx_size ? s->n_tokens : (uint32_t)s->ctx_size;
}
uint32_t layer_rows(const sf37kv_session *s, uint32_t il) {
    uint32_t r = live_rows(s);
    const uint32_t cap = s->caches[il].cap;
    if (cap != 0 && r > cap) r = cap;
    return r;
}

bool descriptor_ok(const sf37kv_session *s) {
    if (!s || !s->caches) return false;
    const sf37kv_session_layout &L = s->layout;
    if (L.n_layers == 0 || L.n_layers > 4096 || L.kv_heads == 0 || L.head_dim == 0) return false;
    if (s->dtype != SF37KV_F32 && s->dtype != SF37KV_F16) return false;
    return true;
}

uint64_t prefix_bytes(const sf37kv_session *s, uint32_t fields) {
    const sf37kv_session_layout &L = s->layout;
    return (uint64_t)fields * 4u + (uint64_t)L.n_layers * 4u + (uint64_t)s->n_tokens * 4u +
           (uint64_t)L.vocab * 4u + (uint64_t)L.embd * 4u;
}

uint64_t row_sum(const sf37kv_session *s) {
    uint64_t n = 0;
    for (uint32_t il = 0; il < s->layout.n_layers; il++) n += layer_rows(s, il);
    return n;
}

// Header, row counts, tokens, logits, hidden -- the part before the KV rows.
std::vector<uint8_t> build_prefix(const sf37kv_session *s, bool payload) {
    const sf37kv_session_layout &L = s->layout;
    std::vector<uint32_t> w;
    if (!payload) {
        w = {kSnapMagic, kSnapVersion, (uint32_t)s->ctx_size, s->n_tokens, live_rows(s), L.n_layers,
             L.kv_heads, L.head_dim, L.vocab, L.embd, s->backend_kind};
    } else {
        const uint32_t elems = kv_row(L);
        w = {kPayMagic, kPayVersion, (uint32_t)s->ctx_size, s->n_tokens, live_rows(s), L.n_layers,
             L.kv_heads, L.head_dim, L.vocab, L.embd, s->backend_kind, kKvI8Grouped, L.payload_group,
             groups_per_row(elems, L.payload_group), (uint32_t)encoded_row_bytes(elems, L.payload_group)};
    }
    for (uint32_t il = 0; il < L.n_layers; il++) w.push_back(layer_rows(s, il));
    for (uint32_t i = 0; i < s->n_tokens; i++) w.push_back((uint32_t)s->tokens[i]);
    std::vector<uint8_t> out(w.size() * 4u + ((uint64_t)L.vocab + L.embd) * 4u);
    memcpy(out.data(), w.data(), w.size() * 4u);
    memcpy(out.data() + w.size() * 4u, s->logits, (uint64_t)L.vocab * 4u);
    memcpy(out.data() + w.size() * 4u + (uint64_t)L.vocab * 4u, s->hidden, (uint64_t)L.embd * 4u);
    return out;
}

// Pack descriptors of every layer's live rows, sections back to back.
std::vector<sf37kv_pack_layer> kv_sections(const sf37kv_session *s, const uint32_t *rows, uint32_t tokens,
                                           uint64_t row_bytes) {
    std::vector<sf37kv_pack_layer> v(s->layout.n_layers);
    uint64_t off = 0;
    for (uint32_t il = 0; il < s->layout.n_layers; il++) {
        v[il].cache = s->caches[il];
        v[il].first_pos = tokens - rows[il];
        v[il].rows = rows[il];
        v[il].offset = off;
        off += 2ull * rows[il] * row_bytes;
    }
    return v;
}

// ------------------------------------------------------------ header checks
// The loaders' validation, in the reference's order.  h: header words;
// rows: row counts.  fields 11 = snapshot, 15 = payload.
int check_header(const sf37kv_session *s, const uint32_t *h, const uint32_t *rows, bool payload,
                 char *err, size_t errlen) {
    const sf37kv_session_layout &L = s->layout;
    const char *what = payload ? "session payload" : "session snapshot";
    const uint32_t saved_ctx = h[2], token_count = h[3], live = h[4];
    if (!payload) {
        // sf37.c:7375-7387
        if (saved_ctx != (uint32_t)s->ctx_size)
            return fail(err, errlen, "session snapshot ctx %u does not match current ctx %d", saved_ctx,
                        s->ctx_size);
        if (token_count > (uint32_t)s->ctx_size || live > token_count ||
            live != (token_count < saved_ctx ? token_count : saved_ctx))
            return fail(err, errlen, "session snapshot has invalid token/cache row counts");
    } else {
        // sf37.c:7067-7075
        if (saved_ctx > (uint32_t)s->ctx_size || token_count > (uint32_t)s->ctx_size)
            return fail(err, errlen, "KV checkpoint does not fit current context");
        if (live > token_count || live != (token_count < saved_ctx ? token_count : saved_ctx))
            return fail(err, errlen, "session payload has invalid token/cache row counts");
    }
    // sf37.c:7388-7410 / 7077-7102
    for (uint32_t il = 0; il < L.n_layers; il++) {
        const uint32_t r = rows[il];
        if (r > live) return fail(err, errlen, "%s has too many KV rows for layer %u", what, il);
        if (layer_full(L, il)) {
            if (r != live) return fail(err, errlen, "%s is missing full-attention KV rows", what);
        } else {
            const uint32_t needed = live < L.sliding_window ? live : L.sliding_window;
            if (r < needed) return fail(err, errlen, "%s is missing sliding-window KV rows", what);
        }
        const uint32_t cap = s->caches[il].cap;
        if (cap != 0 && r > cap) return fail(err, errlen, "%s KV rows do not fit current cache", what);
    }
    // sf37.c:7411-7418 / 7103-7114
    bool layout_ok = h[5] == L.n_layers && h[6] == L.kv_heads && h[7] == L.head_dim && h[8] == L.vocab &&
                     h[9] == L.embd;
    if (payload) {
        const uint32_t elems = h[6] * h[7];
        layout_ok = layout_ok && h[11] == kKvI8Grouped && h[12] == L.payload_group &&
                    h[13] == groups_per_row(elems, h[12]) && h[14] == encoded_row_bytes(elems, h[12]);
    }
    if (!layout_ok) return fail(err, errlen, "%s was written for a different SF37 layout", what);
    return 0;
}

// ------------------------------------------------------------ fd io
// A file descriptor at a position.  Seekable files (regular files, tmpfs)
// are accessed with pread/pwrite, large transfers split across threads
// (page-cache copies and tmpfs page allocation scale with threads); pipes and
// sockets fall back to sequential read/write.
// A writer to a regular file first extends the file over the record's range
// and maps it, so that the threads copy straight into the page
// cache: parallel pwrite calls on one file serialize on its inode lock.
struct FdIo {
    int fd;
    bool seekable;
    int64_t off;          // next file offset (seekable only)
    uint64_t *remaining;  // loader: bytes of the record not yet read
    char *err;
    size_t errlen;
    bool io_failed = false;  // a callback reported a short read / failed write (message in err)
    uint8_t *map = nullptr;  // writer: mapping of [map_base, map_base + map_len)
    int64_t map_base = 0;
    uint64_t map_len = 0;
};

FdIo fd_io(int fd, uint64_t *remaining, char *err, size_t errlen) {
    const off_t o = lseek(fd, 0, SEEK_CUR);
    return FdIo{fd, o >= 0, (int64_t)o, remaining, err, errlen};
}

// Maps [off, off + bytes) of a regular file for writing; silently keeps the
// pwrite path when the file system cannot allocate or map.
void fd_map_for_write(FdIo &io, uint64_t bytes) {
    struct stat st;
    if (!io.seekable || bytes < (64ull << 20) || fstat(io.fd, &st) != 0 || !S_ISREG(st.st_mode)) return;
    // extend (sparse) rather than fallocate: the pages are then allocated by
    // the copying threads' faults, in parallel
    const off_t end = (off_t)io.off + (off_t)bytes;
    if (st.st_size < end && ftruncate(io.fd, end) != 0) return;
    const int64_t base = io.off & ~(int64_t)4095;
    const uint64_t len = bytes + (uint64_t)(io.off - base);
    void *m = mmap(nullptr, len, PROT_READ | PROT_WRITE, MAP_SHARED, io.fd, (off_t)base);
    if (m == MAP_FAILED) return;
    io.map = (uint8_t *)m;
    io.map_base = base;
    io.map_len = len;
}

// Ends a call: unmaps, and leaves a seekable fd at the end of what was
// transferred, as sequential I/O would.
void fd_done(FdIo &io) {
    if (io.map) {
        munmap(io.map, io.map_len);
        io.map = nullptr;
    }
    if (io.seekable) (void)lseek(io.fd, (off_t)io.off, SEEK_SET);
}

int seq_io(int fd, uint8_t *b, uint64_t n, bool wr) {
    while (n > 0) {
        const size_t c = n > kIoChunk ? (size_t)kIoChunk : (size_t)n;
        const ssize_t r = wr ? write(fd, b, c) : read(fd, b, c);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return 1;
        b += r;
        n -= (uint64_t)r;
    }
    return 0;
}

int pos_io(int fd, uint8_t *b, uint64_t n, int64_t off, bool wr) {
    while (n > 0) {
        const size_t c = n > kIoChunk ? (size_t)kIoChunk : (size_t)n;
        const ssize_t r = wr ? pwrite(fd, b, c, (off_t)off) : pread(fd, b, c, (off_t)off);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return 1;
        b += r;
        off += r;
        n -= (uint64_t)r;
    }
    return 0;
}

int par_io(FdIo &io, void *p, uint64_t n, bool wr) {
    uint8_t *b = (uint8_t *)p;
    if (!io.seekable) return seq_io(io.fd, b, n, wr);
    constexpr uint64_t kMinPart = 4ull << 20;
    unsigned nt = std::thread::hardware_concurrency();
    nt = nt < 1 ? 1 : nt > 8 ? 8 : nt;
    if (n < 2 * kMinPart || nt == 1) {
        const int rc = pos_io(io.fd, b, n, io.off, wr);
        if (!rc) io.off += (int64_t)n;
        return rc;
    }
    if ((uint64_t)nt > n / kMinPart) nt = (unsigned)(n / kMinPart);
    const uint64_t part = ((n + nt - 1) / nt + 4095) & ~4095ull;
    const bool mapped = wr && io.map && io.off >= io.map_base &&
                        (uint64_t)(io.off - io.map_base) + n <= io.map_len;
    std::atomic<int> bad{0};
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; t++) {
        const uint64_t a = (uint64_t)t * part;
        if (a >= n) break;
        const uint64_t len = n - a < part ? n - a : part;
        th.emplace_back([&, a, len] {
            if (mapped) memcpy(io.map + (io.off - io.map_base) + a, b + a, len);
            else if (pos_io(io.fd, b + a, len, io.off + (int64_t)a, wr)) bad = 1;
        });
    }
    for (auto &x : th) x.join();
    if (!bad) io.off += (int64_t)n;
    return bad.load();
}

int sink_fd(const void *p, uint64_t n, void *ctx) {
    FdIo *S = (FdIo *)ctx;
    if (par_io(*S, const_cast<void *>(p), n, true)) {
        S->io_failed = true;
        return fail(S->err, S->errlen, "failed to write session payload");
    }
    return 0;
}

// payload_read_bytes (sf37.c:6753-6772): fails on a short file or when the
// record's byte budget is exhausted.
int source_fd(void *p, uint64_t n, void *ctx) {
    FdIo *S = (FdIo *)ctx;
    if (n > *S->remaining || par_io(*S, p, n, false)) {
        S->io_failed = true;
        return fail(S->err, S->errlen, "truncated session payload");
    }
    *S->remaining -= n;
    return 0;
}

}  // namespace
}  // namespace sf37kv

using namespace sf37kv;

extern "C" sf37kv_session_layout sf37kv_session_layout_default(void) {
    sf37kv_session_layout L;
    L.n_layers = 45;
    L.kv_heads = 8;
    L.head_dim = 128;
    L.vocab = 128896;
    L.embd = 4096;
    L.sliding_window = 512;
    L.full_every = 4;
    L.payload_group = 64;
    return L;
}

extern "C" uint64_t sf37kv_session_snapshot_bytes(const sf37kv_session *s) {
    if (!descriptor_ok(s)) return 0;
    return prefix_bytes(s, kSnapFields) + row_sum(s) * 2ull * kv_row(s->layout) * 4u;
}

extern "C" uint64_t sf37kv_session_payload_bytes(const sf37kv_session *s) {
    if (!descriptor_ok(s)) return 0;
    return prefix_bytes(s, kPayFields) +
           row_sum(s) * 2ull * encoded_row_bytes(kv_row(s->layout), s->layout.payload_group);
}

extern "C" int sf37kv_session_save_snapshot(const sf37kv_session *s, void *dst, uint64_t dst_cap, uint64_t *len,
                                            char *err, size_t errlen) {
    if (!descriptor_ok(s) || !dst || (s->n_tokens && !s->tokens) || !s->logits || !s->hidden)
        return fail(err, errlen, "session has no valid checkpoint to snapshot");
    const uint64_t bytes = sf37kv_session_snapshot_bytes(s);
    if (dst_cap < bytes) return fail(err, errlen, "session snapshot writer overflow");
    const std::vector<uint8_t> pre = build_prefix(s, false);
    memcpy(dst, pre.data(), pre.size());
    const uint32_t L = s->layout.n_layers;
    std::vector<uint32_t> rows(L);
    for (uint32_t il = 0; il < L; il++) rows[il] = layer_rows(s, il);
    const auto sec = kv_sections(s, rows.data(), s->n_tokens, (uint64_t)kv_row(s->layout) * 4u);
    if (sf37kv_pack_to_host((uint8_t *)dst + pre.size(), sec.data(), L, kv_row(s->layout), s->dtype,
                            SF37KV_FMT_RAW_F32, 0, 1))
        return fail_last(err, errlen, "failed to read CUDA KV cache for snapshot");
    if (len) *len = bytes;
    return 0;
}

extern "C" int sf37kv_session_load_snapshot(sf37kv_session *s, const void *src, uint64_t len, char *err,
                                            size_t errlen) {
    if (!descriptor_ok(s) || !src || len == 0 || !s->tokens || !s->logits || !s->hidden)
        return fail(err, errlen, "invalid session snapshot load");
    const sf37kv_session_layout &L = s->layout;
    const uint8_t *p = (const uint8_t *)src;
    uint64_t pos = 0;
    auto take = [&](void *d, uint64_t n) -> bool {
        if (n > len || pos > len - n) return false;
        memcpy(d, p + pos, n);
        pos += n;
        return true;
    };
    uint32_t h[kSnapFields];
    if (!take(h, sizeof(h))) return fail(err, errlen, "truncated session snapshot header");
    if (h[0] != kSnapMagic || h[1] != kSnapVersion) return fail(err, errlen, "unsupported session snapshot version");
    std::vector<uint32_t> rows(L.n_layers);
    if (!take(rows.data(), (uint64_t)L.n_layers * 4u))
        return fail(err, errlen, "truncated session snapshot KV row counts");
    if (check_header(s, h, rows.data(), false, err, errlen)) return 1;
    const uint32_t token_count = h[3];
    std::vector<uint32_t> toks(token_count);
    for (uint32_t i = 0; i < token_count; i++)
        if (!take(&toks[i], 4) || toks[i] >= L.vocab)
            return fail(err, errlen, "session snapshot has invalid token data");
    if (!take(s->logits, (uint64_t)L.vocab * 4u) || !take(s->hidden, (uint64_t)L.embd * 4u))
        return fail(err, errlen, "truncated session snapshot logits/hidden");
    uint64_t kv_bytes = 0;
    const uint64_t rb = (uint64_t)kv_row(L) * 4u;
    for (uint32_t il = 0; il < L.n_layers; il++) kv_bytes += 2ull * rows[il] * rb;
    if (kv_bytes > len - pos) return fail(err, errlen, "failed to restore CUDA KV cache from snapshot");
    // checked before any cache write (the reference checks after restoring)
    if (pos + kv_bytes != len) return fail(err, errlen, "session snapshot has trailing bytes");
    const auto sec = kv_sections(s, rows.data(), token_count, rb);
    if (sf37kv_unpack_from_host(p + pos, sec.data(), L.n_layers, kv_row(L), s->dtype, SF37KV_FMT_RAW_F32, 0))
        return fail_last(err, errlen, "failed to restore CUDA KV cache from snapshot");
    for (uint32_t i = 0; i < token_count; i++) s->tokens[i] = (int32_t)toks[i];
    s->n_tokens = token_count;
    return 0;
}

extern "C" int sf37kv_session_save_payload(const sf37kv_session *s, int fd, char *err, size_t errlen) {
    if (!descriptor_ok(s) || fd < 0 || (s->n_tokens && !s->tokens) || !s->logits || !s->hidden)
        return fail(err, errlen, "session has no valid checkpoint to save");
    if (err && errlen) err[0] = 0;
    const sf37kv_session_layout &L = s->layout;
    const std::vector<uint8_t> pre = build_prefix(s, true);
    FdIo io = fd_io(fd, nullptr, err, errlen);
    fd_map_for_write(io, sf37kv_session_payload_bytes(s));
    if (sink_fd(pre.data(), pre.size(), &io)) {
        fd_done(io);
        return 1;
    }
    std::vector<uint32_t> rows(L.n_layers);
    for (uint32_t il = 0; il < L.n_layers; il++) rows[il] = layer_rows(s, il);
    const uint64_t rb = encoded_row_bytes(kv_row(L), L.payload_group);
    const auto sec = kv_sections(s, rows.data(), s->n_tokens, rb);
    const int rc = pack_stream(sec.data(), L.n_layers, kv_row(L), s->dtype, SF37KV_FMT_I8_GROUPED, L.payload_group,
                               sink_fd, &io);
    fd_done(io);
    if (rc && io.io_failed) return 1;  // the sink's message
    if (rc) return fail_last(err, errlen, "failed to read CUDA K cache for payload");
    return 0;
}

namespace sf37kv {
namespace {
int load_payload_body(sf37kv_session *s, FdIo &src, uint64_t payload_bytes, char *err, size_t errlen) {
    const sf37kv_session_layout &L = s->layout;
    uint64_t &remaining = *src.remaining;
    uint32_t h[kPayFields];
    if (source_fd(h, sizeof(h), &src)) return 1;
    if (h[0] != kPayMagic || h[1] != kPayVersion) return fail(err, errlen, "unsupported session payload version");
    std::vector<uint32_t> rows(L.n_layers);
    if (source_fd(rows.data(), (uint64_t)L.n_layers * 4u, &src)) return 1;
    if (check_header(s, h, rows.data(), true, err, errlen)) return 1;
    const uint32_t token_count = h[3];
    const uint64_t rb = encoded_row_bytes(kv_row(L), L.payload_group);
    uint64_t sum = 0;
    for (uint32_t il = 0; il < L.n_layers; il++) sum += rows[il];
    const uint64_t expected = (uint64_t)kPayFields * 4u + (uint64_t)L.n_layers * 4u + (uint64_t)token_count * 4u +
                              (uint64_t)L.vocab * 4u + (uint64_t)L.embd * 4u + sum * 2u * rb;
    if (payload_bytes != expected) return fail(err, errlen, "session payload byte count mismatch");
    std::vector<uint32_t> toks(token_count);
    if (token_count && (source_fd(toks.data(), (uint64_t)token_count * 4u, &src)))
        return fail(err, errlen, "session payload has invalid token data");
    for (uint32_t i = 0; i < token_count; i++)
        if (toks[i] >= L.vocab) return fail(err, errlen, "session payload has invalid token data");
    if (source_fd(s->logits, (uint64_t)L.vocab * 4u, &src) || source_fd(s->hidden, (uint64_t)L.embd * 4u, &src))
        return 1;
    const auto sec = kv_sections(s, rows.data(), token_count, rb);
    const int rc = unpack_stream(sec.data(), L.n_layers, kv_row(L), s->dtype, SF37KV_FMT_I8_GROUPED,
                                 L.payload_group, source_fd, &src);
    if (rc && src.io_failed) return 1;  // the source's message
    if (rc) return fail_last(err, errlen, "failed to restore CUDA K cache from payload");
    if (remaining != 0) return fail(err, errlen, "session payload has trailing bytes");
    for (uint32_t i = 0; i < token_count; i++) s->tokens[i] = (int32_t)toks[i];
    s->n_tokens = token_count;
    return 0;
}
}  // namespace
}  // namespace sf37kv

extern "C" int sf37kv_session_load_payload(sf37kv_session *s, int fd, uint64_t payload_bytes, char *err,
                                           size_t errlen) {
    if (!descriptor_ok(s) || fd < 0 || payload_bytes == 0 || !s->tokens || !s->logits || !s->hidden)
        return fail(err, errlen, "invalid session payload load");
    if (err && errlen) err[0] = 0;
    uint64_t remaining = payload_bytes;
    FdIo src = fd_io(fd, &remaining, err, errlen);
    const int rc = load_payload_body(s, src, payload_bytes, err, errlen);
    fd_done(src);
    return rc;
}
