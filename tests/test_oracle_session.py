"""CPU: the session checkpoint restatement (oracle/session.py) pinned
against the reference's own writers and loaders -- the committed golden
bytes and messages, and the live reference library (oracle/_ref) when it is
built."""
import os

import numpy as np
import pytest

import oracle
from oracle import session as S
from tests import session_cases as C

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sessions.npz")
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def _tie_only_diffs(mine, ref, prefix, src, kv=C.KV, group=64):
    """Payload bytes may differ only in int8 codes of values whose quotient
    x / scale lies on a .5 tie: the reference's vectorized division under
    -ffast-math uses the CPU's reciprocal estimate (rcpps + one Newton step),
    whose last bit is hardware-specific.  Everything else is exact.
    src: the f32 source rows in payload order."""
    a = np.frombuffer(mine, np.uint8)
    b = np.frombuffer(ref, np.uint8)
    assert a.size == b.size
    d = np.nonzero(a != b)[0]
    assert np.all(d >= prefix), "header/tokens/logits/hidden differ"
    ns = kv // group
    rb = ns * 4 + kv
    rows = (d - prefix) // rb
    col = (d - prefix) % rb
    assert np.all(col >= ns * 4), "a group scale differs"
    qa, qb = a[d].view(np.int8).astype(int), b[d].view(np.int8).astype(int)
    assert np.all(np.abs(qa - qb) == 1)
    enc = a[prefix:].reshape(-1, rb)
    el = col - ns * 4
    for k in range(rows.size):
        s = float(enc[rows[k], 4 * (el[k] // group):4 * (el[k] // group) + 4].view(np.float32)[0])
        t = float(src[rows[k], el[k]]) / s
        assert abs(abs(t - np.trunc(t)) - 0.5) < 1e-5 * max(1.0, abs(t)), (rows[k], el[k], t)
    return d.size


def _payload_src(kc, vc, n, ctx, caps):
    rows = S.layer_rows(n, ctx, caps)
    out = []
    for il in range(C.LAYERS):
        k = C.live_rows_in_order(kc[il], n, rows[il], caps[il])
        v = C.live_rows_in_order(vc[il], n, rows[il], caps[il])
        out.append(np.stack([k, v], 1).reshape(-1, C.KV))
    return np.concatenate(out)


def _snap_prefix(n_tokens, kind):
    return (11 if kind == 0 else 15) * 4 + (C.LAYERS + n_tokens + C.VOCAB + C.EMBD) * 4


@pytest.mark.parametrize("kind", [0, 1])
def test_oracle_writer_matches_reference_golden(kind):
    g = np.load(GOLD)
    ctx, n = 3, 2
    toks, lg, hd, kc, vc = C.state(7, ctx, n, [ctx] * C.LAYERS, coarse=True)
    mine = S.save(kind, ctx, toks, lg, hd, kc, vc, [ctx] * C.LAYERS, backend=0)
    ref = g["snapshot" if kind == 0 else "payload"].tobytes()
    if kind == 0:
        mine = S.cpu_layout_snapshot(mine, C.LAYERS, S.layer_rows(n, ctx, [ctx] * C.LAYERS))
        assert mine == ref
    else:
        _tie_only_diffs(mine, ref, _snap_prefix(n, 1), _payload_src(kc, vc, n, ctx, [ctx] * C.LAYERS))


def test_oracle_loader_messages_match_reference_golden():
    g = np.load(GOLD)
    want = dict(zip(g["names"].tolist(), g["msgs"].tolist()))
    ctx = 3
    for kind in (0, 1):
        buf = g["snapshot" if kind == 0 else "payload"].tobytes()
        for name, bad, lctx in C.corruptions(kind, buf, ctx):
            kc = [np.zeros((ctx, C.KV), np.float32) for _ in range(C.LAYERS)]
            vc = [np.zeros((ctx, C.KV), np.float32) for _ in range(C.LAYERS)]
            with pytest.raises(S.LoadError) as e:
                S.load(kind, bad, lctx, [ctx] * C.LAYERS, kc, vc)
            ref = want[f"{kind}:{name}"]
            if kind == 0 and name == "truncated_kv":
                # the CPU backend's wording; the CUDA-backend loader (restated
                # here) says sf37.c:7453's message instead
                assert ref == "truncated CPU KV cache in session snapshot"
                assert str(e.value) == "failed to restore CUDA KV cache from snapshot"
            else:
                assert str(e.value) == ref, name


def test_oracle_loader_reads_reference_payload():
    g = np.load(GOLD)
    ctx, n = 3, 2
    toks, lg, hd, kc, vc = C.state(7, ctx, n, [ctx] * C.LAYERS, coarse=True)
    k2 = [np.zeros_like(k) for k in kc]
    v2 = [np.zeros_like(v) for v in vc]
    t, l, h = S.load(1, g["payload"].tobytes(), ctx, [ctx] * C.LAYERS, k2, v2)
    assert np.array_equal(t, toks) and np.array_equal(l, lg) and np.array_equal(h, hd)
    for il in range(C.LAYERS):
        for p in range(n):
            assert np.abs(k2[il][p] - kc[il][p]).max() <= np.abs(kc[il][p]).max() / 127 * 0.5 + 1e-7


@needs_ref
@pytest.mark.parametrize("kind", [0, 1])
def test_oracle_ring_session_matches_live_reference(kind):
    # 530 tokens in a 544 context; sliding layers keep 520 rows in a 520-slot
    # ring (>= the 512 window), full layers all 530: ring wrap + per-layer
    # row counts.
    ctx, n = 544, 530
    caps = [ctx if il % 4 == 0 else 520 for il in range(C.LAYERS)]
    toks, lg, hd, kc, vc = C.state(11, ctx, n, caps, f16=True)
    rows = S.layer_rows(n, ctx, caps)
    mine = S.save(kind, ctx, toks, lg, hd, kc, vc, caps, backend=0)
    kr = [C.live_rows_in_order(kc[i], n, rows[i], caps[i]) for i in range(C.LAYERS)]
    vr = [C.live_rows_in_order(vc[i], n, rows[i], caps[i]) for i in range(C.LAYERS)]
    ref = S.ref_session_save(kind, ctx, toks, lg, hd, kr, vr)
    if kind == 0:
        assert S.cpu_layout_snapshot(mine, C.LAYERS, rows) == ref
    else:
        _tie_only_diffs(mine, ref, _snap_prefix(n, 1), _payload_src(kc, vc, n, ctx, caps))
        # and the reference loader restores our bytes to what the oracle decodes
        t, l, h, kk, vv = S.ref_session_load(1, mine, ctx)
        assert np.array_equal(t, toks) and [k.shape[0] for k in kk] == rows
        k2 = [np.zeros((c, C.KV), np.float32) for c in caps]
        v2 = [np.zeros((c, C.KV), np.float32) for c in caps]
        S.load(1, mine, ctx, caps, k2, v2)
        for il in (0, 1, 44):
            assert np.array_equal(kk[il], C.live_rows_in_order(k2[il], n, rows[il], caps[il]))
            assert np.array_equal(vv[il], C.live_rows_in_order(v2[il], n, rows[il], caps[il]))


@pytest.mark.parametrize("kind", [0, 1])
def test_head_slices_tile_the_record_rows(kind):
    # The N slices' byte ranges of a row are disjoint and cover it, and the
    # bytes a slice's own (narrower) row encodes are the record row's bytes
    # at those ranges: packing per KV-head slice needs no exchange.
    rng = np.random.default_rng(4)
    k = rng.standard_normal((6, 1024)).astype(np.float32)
    v = rng.standard_normal((6, 1024)).astype(np.float32)
    full = oracle.pack_layer(k, v, 0, 6, 6, 1024, fmt=kind).reshape(12, -1)
    rb = full.shape[1]
    for n in (1, 2, 4, 8):
        w = 1024 // n
        cover = np.zeros(rb, np.int32)
        for r in range(n):
            rngs = S.slice_columns(kind, col0=r * w, width=w)
            part = oracle.pack_layer(np.ascontiguousarray(k[:, r * w:(r + 1) * w]),
                                     np.ascontiguousarray(v[:, r * w:(r + 1) * w]), 0, 6, 6, w, fmt=kind).reshape(12, -1)
            pos = 0
            for start, length in rngs:
                cover[start:start + length] += 1
                assert np.array_equal(full[:, start:start + length], part[:, pos:pos + length])
                pos += length
            assert pos == part.shape[1]
        assert np.all(cover == 1)
