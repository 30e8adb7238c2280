"""Seeded session states and corrupted checkpoints shared by the session
tests and the golden-fixture generator (host-only helpers)."""
import numpy as np

LAYERS, KV, VOCAB, EMBD = 45, 1024, 128896, 4096


def state(seed, ctx, n_tokens, caps, coarse=False, f16=False):
    """tokens, logits, hidden, and per-layer ring caches [cap][1024] (f32, or
    uint16 f16 bits) whose slots hold position p at p % cap.  coarse: values
    on a 1/2 grid (compressible fixtures)."""
    rng = np.random.default_rng(seed)
    tokens = rng.integers(0, VOCAB, n_tokens).astype(np.int32)
    logits = rng.standard_normal(VOCAB).astype(np.float32)
    hidden = rng.standard_normal(EMBD).astype(np.float32)
    if coarse:
        logits = np.round(logits * 2) / 2
        hidden = np.round(hidden * 2) / 2
    kc, vc = [], []
    for c in caps:
        k = rng.standard_normal((c, KV)).astype(np.float32)
        v = rng.standard_normal((c, KV)).astype(np.float32)
        if coarse:
            k, v = np.round(k * 2) / 2, np.round(v * 2) / 2
        if f16:
            k, v = k.astype(np.float16).view(np.uint16), v.astype(np.float16).view(np.uint16)
        kc.append(k)
        vc.append(v)
    return tokens, logits.astype(np.float32), hidden.astype(np.float32), kc, vc


def live_rows_in_order(cache, n_tokens, rows, cap):
    """The rows of positions n_tokens-rows .. n_tokens-1 as f32 [rows][1024]."""
    idx = [(n_tokens - rows + r) % cap for r in range(rows)]
    c = cache[idx]
    return c.view(np.float16).astype(np.float32) if c.dtype == np.uint16 else c


def corruptions(kind, buf, ctx):
    """(name, bytes, load ctx) variants of a valid checkpoint that the
    loaders must reject, one per check."""
    nf = 11 if kind == 0 else 15
    b = bytes(buf)

    def word(i, v):
        x = bytearray(b)
        x[4 * i:4 * i + 4] = np.array([v], "<u4").tobytes()
        return bytes(x)

    h = np.frombuffer(b[:4 * nf], "<u4")
    rows0 = 4 * nf
    tok0 = rows0 + 4 * LAYERS
    out = [
        ("magic", word(0, 0x12345678), ctx),
        ("version", word(1, 9), ctx),
        ("short_header", b[:4 * nf - 4], ctx),
        ("short_rows", b[:rows0 + 8], ctx),
        ("ctx", b, ctx - 1),
        ("tokens_gt_ctx", word(3, ctx + 5), ctx),
        ("live_mismatch", word(4, int(h[4]) - 1), ctx),
        ("too_many_rows", word(nf + 1, int(h[4]) + 1), ctx),
        ("full_missing", word(nf + 0, int(h[4]) - 1), ctx),
        ("sliding_missing", word(nf + 1, 0), ctx),
        ("layout_layers", word(5, LAYERS + 1), ctx),
        ("layout_vocab", word(8, VOCAB - 1), ctx),
        ("bad_token", word(nf + LAYERS, VOCAB), ctx),
        ("truncated_kv", b[:-16], ctx),
        ("trailing", b + b"\0" * 8, ctx),
        ("short_logits", b[:tok0 + 4 * int(h[3]) + 100], ctx),
    ]
    if kind == 1:
        out += [("layout_group", word(12, 32), ctx), ("layout_enc", word(11, 2), ctx)]
    return out
