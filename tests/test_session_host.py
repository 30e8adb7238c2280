"""CPU: the library's session loaders (C ABI) reject every corrupted
checkpoint with the reference's message before touching a cache, and the
size queries match the formats (no GPU: the caches are never reached)."""
import ctypes
import os
import tempfile

import numpy as np
import pytest

from sf37_b200 import _lib
from tests import session_cases as C

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sessions.npz")


def _session(ctx, n_tokens=0, caps=None, dtype=4):
    L = _lib.lib().sf37kv_session_layout_default()
    caches = (_lib.Cache * C.LAYERS)()
    for i in range(C.LAYERS):
        caches[i] = _lib.Cache(0x1000, 0x2000, (caps or [ctx] * C.LAYERS)[i], 0, 0, 0)
    keep = dict(tokens=np.zeros(max(ctx, n_tokens, 1), np.int32), logits=np.zeros(C.VOCAB, np.float32),
                hidden=np.zeros(C.EMBD, np.float32), caches=caches)
    s = _lib.Session(L, ctx, n_tokens, keep["tokens"].ctypes.data, keep["logits"].ctypes.data,
                     keep["hidden"].ctypes.data, caches, dtype, 1)
    return s, keep


def test_layout_default_is_the_reference_model():
    L = _lib.lib().sf37kv_session_layout_default()
    assert (L.n_layers, L.kv_heads, L.head_dim, L.vocab, L.embd, L.sliding_window, L.full_every,
            L.payload_group) == (45, 8, 128, 128896, 4096, 512, 4, 64)


def test_byte_counts_match_formats():
    # sf37.c:6809-6835: 32768 tokens in a 32768 context, every layer full cap
    s, _ = _session(32768, 32768)
    base = (C.LAYERS + 32768 + C.VOCAB + C.EMBD) * 4
    assert _lib.lib().sf37kv_session_snapshot_bytes(ctypes.byref(s)) == 11 * 4 + base + 45 * 32768 * 8192
    assert _lib.lib().sf37kv_session_payload_bytes(ctypes.byref(s)) == 15 * 4 + base + 45 * 32768 * 2 * 1088
    # ring caps clamp the sliding layers' rows
    caps = [32768 if il % 4 == 0 else 8192 for il in range(C.LAYERS)]
    s, _ = _session(32768, 30000, caps)
    rows = sum(min(30000, c) for c in caps)
    assert _lib.lib().sf37kv_session_payload_bytes(ctypes.byref(s)) == \
        15 * 4 + (C.LAYERS + 30000 + C.VOCAB + C.EMBD) * 4 + rows * 2 * 1088


@pytest.mark.parametrize("kind", [0, 1])
def test_loader_messages_match_reference_golden(kind):
    g = np.load(GOLD)
    want = dict(zip(g["names"].tolist(), g["msgs"].tolist()))
    buf = g["snapshot" if kind == 0 else "payload"].tobytes()
    L = _lib.lib()
    for name, bad, lctx in C.corruptions(kind, buf, 3):
        s, keep = _session(lctx)
        err = ctypes.create_string_buffer(512)
        if kind == 0:
            arr = np.frombuffer(bad, np.uint8)
            rc = L.sf37kv_session_load_snapshot(ctypes.byref(s), arr.ctypes.data, arr.size, err, 512)
        else:
            with tempfile.TemporaryFile() as f:
                f.write(bad)
                f.flush()
                f.seek(0)
                rc = L.sf37kv_session_load_payload(ctypes.byref(s), f.fileno(), len(bad), err, 512)
                if name in ("truncated_kv", "trailing", "short_logits"):
                    assert os.lseek(f.fileno(), 0, os.SEEK_CUR) > 0  # the header was consumed
        assert rc == 1, name
        ref = want[f"{kind}:{name}"]
        if kind == 0 and name == "truncated_kv":
            ref = "failed to restore CUDA KV cache from snapshot"  # the CUDA backend's wording
        assert err.value.decode() == ref, name
        assert _lib.last_error() == ref
        del keep


def test_payload_write_error_reports_reference_message():
    s, keep = _session(4, 3)
    r, w = os.pipe()
    os.close(r)  # writing to a pipe without a reader fails (EPIPE)
    import signal
    old = signal.signal(signal.SIGPIPE, signal.SIG_IGN)
    try:
        err = ctypes.create_string_buffer(256)
        assert _lib.lib().sf37kv_session_save_payload(ctypes.byref(s), w, err, 256) == 1
        assert err.value.decode() == "failed to write session payload"
    finally:
        signal.signal(signal.SIGPIPE, old)
        os.close(w)


@pytest.mark.parametrize("kind", [0, 1])
def test_random_header_corruptions_agree_with_oracle(kind):
    # Random single-word corruptions of the reference's golden records
    # (header, row counts, tokens) and random truncations / extensions: every
    # one the oracle loader rejects, the library rejects with the same words,
    # before touching a cache.
    from oracle import session as S
    g = np.load(GOLD)
    buf = g["snapshot" if kind == 0 else "payload"].tobytes()
    nf = 11 if kind == 0 else 15
    n_words = nf + C.LAYERS + 2
    rng = np.random.default_rng(40 + kind)
    L = _lib.lib()
    checked = 0
    for trial in range(300):
        b = bytearray(buf)
        op = rng.integers(0, 3)
        if op == 0:
            w = int(rng.integers(0, n_words))
            val = int(rng.choice([0, 1, 2, 3, 4, 511, 512, 513, 2**31, 2**32 - 1, int(rng.integers(0, 2**32))]))
            b[4 * w:4 * w + 4] = np.array([val], "<u4").tobytes()
        elif op == 1:
            b = b[:int(rng.integers(0, len(b)))]
        else:
            b = b + bytes(int(rng.integers(1, 64)))
        b = bytes(b)
        if not b:
            continue
        try:
            kc = [np.zeros((3, C.KV), np.float32) for _ in range(C.LAYERS)]
            S.load(kind, b, 3, [3] * C.LAYERS, kc, [k.copy() for k in kc])
            continue  # accepted by the oracle: restoring needs the GPU
        except S.LoadError as e:
            want = str(e)
        except (ValueError, IndexError):
            continue
        s, keep = _session(3)
        err = ctypes.create_string_buffer(512)
        if kind == 0:
            arr = np.frombuffer(b, np.uint8)
            rc = L.sf37kv_session_load_snapshot(ctypes.byref(s), arr.ctypes.data, arr.size, err, 512)
        else:
            with tempfile.TemporaryFile() as f:
                f.write(b)
                f.flush()
                f.seek(0)
                rc = L.sf37kv_session_load_payload(ctypes.byref(s), f.fileno(), len(b), err, 512)
        assert rc == 1
        assert err.value.decode() == want, (trial, op, want)
        checked += 1
    assert checked > 100
