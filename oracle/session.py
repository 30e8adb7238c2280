"""Session checkpoint formats, restated with numpy -- TEST INFRASTRUCTURE ONLY.

The raw snapshot (format 2) and the int8-grouped payload (format 3) that the
reference writes from a CUDA session, and the checks its loaders make, in
the reference's order and wording:

  writer   sf37_session_save_snapshot  sf37.c:7235-7345
           sf37_session_save_payload   sf37.c:6922-7036
  loader   sf37_session_load_snapshot  sf37.c:7347-7500
           sf37_session_load_payload   sf37.c:7038-7233
  rows     session_live_kv_rows / session_layer_live_kv_rows  sf37.c:6495-6521

The KV rows are formed by this package's pack_layer (the CUDA-backend row
order: per live position, the K row then the V row).  Pinned against the
reference's own writers and loaders through oracle/_ref (ref_session_save /
ref_session_load below), which run a CPU-backend session.
"""
import ctypes
import tempfile

import numpy as np

from . import _ptr, pack_layer, payload_row_bytes, ref, unpack_layer

SNAP_MAGIC, SNAP_VERSION = 0x37334653, 2
PAY_MAGIC, PAY_VERSION = 0x37375053, 3
LAYOUT = dict(n_layers=45, kv_heads=8, head_dim=128, vocab=128896, embd=4096, sliding_window=512,
              full_every=4, group=64)


def live_rows(n_tokens, ctx):
    return 0 if n_tokens <= 0 or ctx <= 0 else min(n_tokens, ctx)


def layer_rows(n_tokens, ctx, caps):
    live = live_rows(n_tokens, ctx)
    return [min(live, c) if c else live for c in caps]


def _prefix(kind, ctx, tokens, logits, hidden, caps, backend, L):
    kv = L["kv_heads"] * L["head_dim"]
    g = L["group"]
    groups = (kv + g - 1) // g
    head = [SNAP_MAGIC, SNAP_VERSION] if kind == 0 else [PAY_MAGIC, PAY_VERSION]
    head += [ctx, len(tokens), live_rows(len(tokens), ctx), L["n_layers"], L["kv_heads"], L["head_dim"],
             L["vocab"], L["embd"], backend]
    if kind == 1:
        head += [1, g, groups, groups * 4 + kv]
    words = np.array(head + layer_rows(len(tokens), ctx, caps) + list(tokens), dtype="<u4")
    return (words.tobytes() + np.asarray(logits, "<f4").tobytes() + np.asarray(hidden, "<f4").tobytes())


def save(kind, ctx, tokens, logits, hidden, k_caches, v_caches, caps, backend=1, layout=LAYOUT):
    """Bytes of a checkpoint of kind 0 (raw snapshot) or 1 (payload).
    k_caches[il] / v_caches[il]: [cap][kv] f32 or uint16 (f16 bits) ring caches."""
    L = layout
    kv = L["kv_heads"] * L["head_dim"]
    rows = layer_rows(len(tokens), ctx, caps)
    parts = [_prefix(kind, ctx, tokens, logits, hidden, caps, backend, L)]
    for il in range(L["n_layers"]):
        parts.append(pack_layer(k_caches[il], v_caches[il], len(tokens) - rows[il], rows[il], caps[il], kv,
                                fmt=kind, group=L["group"]).tobytes())
    return b"".join(parts)


class LoadError(Exception):
    pass


def load(kind, buf, ctx, caps, k_caches, v_caches, layout=LAYOUT):
    """Restores buf into the ring caches (in place) after the reference's
    checks.  Returns (tokens, logits, hidden); raises LoadError(message)."""
    L = layout
    buf = bytes(buf)
    what = "session snapshot" if kind == 0 else "session payload"
    pos = 0

    def take(n, msg):
        nonlocal pos
        if n > len(buf) - pos:
            raise LoadError(msg)
        out = buf[pos:pos + n]
        pos += n
        return out

    trunc = "truncated session payload"
    nf = 11 if kind == 0 else 15
    h = np.frombuffer(take(nf * 4, "truncated session snapshot header" if kind == 0 else trunc), "<u4")
    if kind == 0 and (h[0] != SNAP_MAGIC or h[1] != SNAP_VERSION):
        raise LoadError("unsupported session snapshot version")
    if kind == 1 and (h[0] != PAY_MAGIC or h[1] != PAY_VERSION):
        raise LoadError("unsupported session payload version")
    rows = np.frombuffer(take(L["n_layers"] * 4, "truncated session snapshot KV row counts" if kind == 0
                              else trunc), "<u4")
    saved_ctx, token_count, live = int(h[2]), int(h[3]), int(h[4])
    if kind == 0:
        if saved_ctx != ctx:
            raise LoadError(f"session snapshot ctx {saved_ctx} does not match current ctx {ctx}")
        if token_count > ctx or live > token_count or live != min(token_count, saved_ctx):
            raise LoadError("session snapshot has invalid token/cache row counts")
    else:
        if saved_ctx > ctx or token_count > ctx:
            raise LoadError("KV checkpoint does not fit current context")
        if live > token_count or live != min(token_count, saved_ctx):
            raise LoadError("session payload has invalid token/cache row counts")
    for il in range(L["n_layers"]):
        r = int(rows[il])
        if r > live:
            raise LoadError(f"{what} has too many KV rows for layer {il}")
        if il % L["full_every"] == 0:
            if r != live:
                raise LoadError(f"{what} is missing full-attention KV rows")
        elif r < min(live, L["sliding_window"]):
            raise LoadError(f"{what} is missing sliding-window KV rows")
        if caps[il] and r > caps[il]:
            raise LoadError(f"{what} KV rows do not fit current cache")
    ok = (h[5] == L["n_layers"] and h[6] == L["kv_heads"] and h[7] == L["head_dim"] and h[8] == L["vocab"]
          and h[9] == L["embd"])
    kv = int(h[6]) * int(h[7]) if kind == 1 else L["kv_heads"] * L["head_dim"]
    if kind == 1:
        g = int(h[12])
        ok = ok and h[11] == 1 and g == L["group"] and g and h[13] == (kv + g - 1) // g and \
            h[14] == ((kv + g - 1) // g) * 4 + kv
    if not ok:
        raise LoadError(f"{what} was written for a different SF37 layout")
    rb = kv * 4 if kind == 0 else payload_row_bytes(kv, L["group"])
    if kind == 1:
        expected = (15 + L["n_layers"] + token_count + L["vocab"] + L["embd"]) * 4 + int(rows.sum()) * 2 * rb
        if len(buf) != expected:
            raise LoadError("session payload byte count mismatch")
    bad_tok = f"{what} has invalid token data"
    tokens = np.frombuffer(take(token_count * 4, bad_tok), "<u4")
    if np.any(tokens >= L["vocab"]):
        raise LoadError(bad_tok)
    lh = "truncated session snapshot logits/hidden" if kind == 0 else trunc
    logits = np.frombuffer(take(L["vocab"] * 4, lh), "<f4").copy()
    hidden = np.frombuffer(take(L["embd"] * 4, lh), "<f4").copy()
    for il in range(L["n_layers"]):
        r = int(rows[il])
        sec = take(2 * r * rb, "failed to restore CUDA KV cache from snapshot" if kind == 0 else trunc)
        unpack_layer(np.frombuffer(sec, np.uint8), k_caches[il], v_caches[il], token_count - r, r, caps[il],
                     kv, fmt=kind, group=L["group"])
    if pos != len(buf):
        raise LoadError(f"{what} has trailing bytes")
    return tokens.astype(np.int32), logits, hidden


def cpu_layout_snapshot(buf, n_layers, rows, kv=1024):
    """Reorders the KV part of a CUDA-backend raw snapshot (K, V per row) into
    the CPU backend's order (a layer's K rows, then its V rows;
    sf37.c:7322-7336) and sets header word 10 (backend) to 0."""
    b = bytearray(buf)
    b[40:44] = np.array([0], "<u4").tobytes()
    kv_bytes = 2 * sum(rows) * kv * 4
    start = len(b) - kv_bytes
    off = start
    for r in rows:
        sec = np.frombuffer(bytes(b[off:off + 2 * r * kv * 4]), "<f4").reshape(r, 2, kv)
        b[off:off + 2 * r * kv * 4] = np.concatenate([sec[:, 0], sec[:, 1]]).tobytes()
        off += 2 * r * kv * 4
    return bytes(b)


# ------------------------------------------------- the reference's own code
_fpp = ctypes.POINTER(ctypes.c_void_p)


def _bind():
    R = ref()
    if not getattr(R, "_session_bound", False):
        R.sf37ref_session_save.restype = ctypes.c_int64
        R.sf37ref_session_save.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                           ctypes.c_void_p, ctypes.c_void_p, _fpp, _fpp, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_uint64, ctypes.c_char_p, ctypes.c_size_t]
        R.sf37ref_session_load.restype = ctypes.c_int
        R.sf37ref_session_load.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_int,
                                           ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           _fpp, _fpp, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
        R._session_bound = True
    return R


def ref_session_save(kind, ctx, tokens, logits, hidden, k_rows, v_rows):
    """The reference's own writer on a CPU session (45 layers).  k_rows[il]:
    [rows][1024] f32, the layer's live rows in position order.  Returns
    bytes (backend word 0; raw snapshot in the CPU KV order)."""
    R = _bind()
    n = LAYOUT["n_layers"]
    toks = np.ascontiguousarray(tokens, np.int32)
    lg = np.ascontiguousarray(logits, np.float32)
    hd = np.ascontiguousarray(hidden, np.float32)
    ks = [np.ascontiguousarray(k, np.float32) for k in k_rows]
    vs = [np.ascontiguousarray(v, np.float32) for v in v_rows]
    kp = (ctypes.c_void_p * n)(*[k.ctypes.data for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.ctypes.data for v in vs])
    nr = np.array([k.shape[0] for k in ks], np.uint32)
    cap = 64 * 1024 * 1024 + sum(k.nbytes * 2 for k in ks)
    out = np.empty(cap, np.uint8)
    err = ctypes.create_string_buffer(512)
    got = R.sf37ref_session_save(kind, ctx, _ptr(toks), len(toks), _ptr(lg), _ptr(hd), kp, vp, _ptr(nr),
                                 _ptr(out), cap, err, 512)
    if got < 0:
        raise LoadError(err.value.decode())
    return out[:got].tobytes()


def ref_session_load(kind, buf, ctx):
    """The reference's own loader on a CPU session of context ctx.  Returns
    (tokens, logits, hidden, k_rows, v_rows) or raises LoadError(message)."""
    R = _bind()
    n = LAYOUT["n_layers"]
    kv = LAYOUT["kv_heads"] * LAYOUT["head_dim"]
    ks = [np.zeros((ctx, kv), np.float32) for _ in range(n)]
    vs = [np.zeros((ctx, kv), np.float32) for _ in range(n)]
    kp = (ctypes.c_void_p * n)(*[k.ctypes.data for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.ctypes.data for v in vs])
    toks = np.zeros(max(ctx, 1), np.int32)
    ntok = ctypes.c_int(0)
    lg = np.zeros(LAYOUT["vocab"], np.float32)
    hd = np.zeros(LAYOUT["embd"], np.float32)
    nr = np.zeros(n, np.uint32)
    err = ctypes.create_string_buffer(512)
    rc = R.sf37ref_session_load(kind, bytes(buf), len(buf), ctx, _ptr(toks), ctypes.addressof(ntok), _ptr(lg),
                                _ptr(hd), kp, vp, _ptr(nr), err, 512)
    if rc != 0:
        raise LoadError(err.value.decode())
    return (toks[:ntok.value].copy(), lg, hd, [ks[i][:nr[i]] for i in range(n)], [vs[i][:nr[i]] for i in range(n)])


def slice_columns(kind, kv=1024, group=64, col0=0, width=1024):
    """Byte ranges of a KV-head slice (elements [col0, col0 + width)) within
    one full-width record row: [(start, length), ...].  Raw rows are f32
    elements; payload rows are the group scales then the int8 codes
    (payload_encode_kv_row_i8_grouped, sf37.c:6633-6659)."""
    if kind == 0:
        return [(4 * col0, 4 * width)]
    groups = kv // group
    return [(4 * (col0 // group), 4 * (width // group)), (4 * groups + col0, width)]


def ref_kvstore_store(directory, ctx, tokens, logits, hidden, k_rows, v_rows, text):
    """The reference's own sf37_kvstore_store_live_prefix_text on a CPU
    session (45 layers; k_rows[il] the layer's live rows in position order)
    with the cached text given.  Returns the record file's bytes."""
    import hashlib
    import os
    R = ref()
    if not getattr(R, "_kvstore_bound", False):
        R.sf37ref_kvstore_store.restype = ctypes.c_int
        R.sf37ref_kvstore_store.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_void_p, _fpp, _fpp, ctypes.c_void_p,
                                            ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
        R._kvstore_bound = True
    n = LAYOUT["n_layers"]
    toks = np.ascontiguousarray(tokens, np.int32)
    lg = np.ascontiguousarray(logits, np.float32)
    hd = np.ascontiguousarray(hidden, np.float32)
    ks = [np.ascontiguousarray(k, np.float32) for k in k_rows]
    vs = [np.ascontiguousarray(v, np.float32) for v in v_rows]
    kp = (ctypes.c_void_p * n)(*[k.ctypes.data for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.ctypes.data for v in vs])
    nr = np.array([k.shape[0] for k in ks], np.uint32)
    err = ctypes.create_string_buffer(512)
    tb = text.encode() if isinstance(text, str) else bytes(text)
    if not R.sf37ref_kvstore_store(directory.encode(), ctx, _ptr(toks), len(toks), _ptr(lg), _ptr(hd), kp, vp,
                                   _ptr(nr), tb, err, 512):
        raise LoadError(err.value.decode() or "reference kvstore store failed")
    path = os.path.join(directory, hashlib.sha1(tb).hexdigest() + ".kv")
    with open(path, "rb") as f:
        return f.read()
