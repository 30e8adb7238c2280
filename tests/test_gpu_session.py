"""GPU: session checkpoints through the C ABI (sf37kv_session_*) against the
oracle restatement (bit-exact bytes; same loader messages) and the
reference's own payload bytes (golden)."""
import os
import tempfile

import numpy as np
import pytest
import torch

from oracle import session as S
from tests import session_cases as C

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sessions.npz")


def _dev(caches, f16):
    out = []
    for a in caches:
        t = torch.from_numpy(a.view(np.float16) if f16 else a).cuda()
        out.append(t)
    return out


def _session(ctx, caps, kc, vc, f16, toks=None, lg=None, hd=None):
    from sf37_b200.session import Session
    k, v = _dev(kc, f16), _dev(vc, f16)
    s = Session(ctx, list(zip(k, v)))
    if toks is not None:
        s.set_tokens(toks)
        s.logits[:] = lg
        s.hidden[:] = hd
    return s, k, v


def _host(t, f16):
    a = t.cpu().numpy()
    return a.view(np.uint16) if f16 else a


@pytest.mark.parametrize("f16,ctx,n,ring", [(False, 48, 40, False), (True, 544, 530, True)])
def test_snapshot_and_payload_bytes_match_oracle(f16, ctx, n, ring):
    caps = [ctx if (il % 4 == 0 or not ring) else 520 for il in range(C.LAYERS)]
    toks, lg, hd, kc, vc = C.state(3, ctx, n, caps, f16=f16)
    s, _, _ = _session(ctx, caps, kc, vc, f16, toks, lg, hd)
    snap = s.save_snapshot().numpy().tobytes()
    want = S.save(0, ctx, toks, lg, hd, kc, vc, caps)
    assert s.snapshot_bytes() == len(want)
    assert snap == want
    with tempfile.TemporaryFile() as f:
        nb = s.save_payload(f)
        f.seek(0)
        pay = f.read()
    assert nb == len(pay) == s.payload_bytes()
    assert pay == S.save(1, ctx, toks, lg, hd, kc, vc, caps)


@pytest.mark.parametrize("f16", [False, True])
def test_roundtrip_restores_live_slots(f16):
    ctx, n = 544, 530
    caps = [ctx if il % 4 == 0 else 520 for il in range(C.LAYERS)]
    toks, lg, hd, kc, vc = C.state(5, ctx, n, caps, f16=f16)
    s, _, _ = _session(ctx, caps, kc, vc, f16, toks, lg, hd)
    snap = s.save_snapshot().clone()
    with tempfile.TemporaryFile() as f:
        nb = s.save_payload(f)
        zeros = [np.zeros_like(a) for a in kc]
        r, rk, rv = _session(ctx, caps, zeros, [z.copy() for z in zeros], f16)
        r.load_snapshot(snap)
        assert r.n_tokens == n and np.array_equal(r.tokens[:n], toks)
        assert np.array_equal(r.logits, lg) and np.array_equal(r.hidden, hd)
        rows = S.layer_rows(n, ctx, caps)
        for il in range(C.LAYERS):
            for src, dst in ((kc, rk), (vc, rv)):
                got = C.live_rows_in_order(_host(dst[il], f16), n, rows[il], caps[il])
                assert np.array_equal(got, C.live_rows_in_order(src[il], n, rows[il], caps[il]))
        # payload: equal to the oracle's decode of the same bytes
        f.seek(0)
        p, pk, pv = _session(ctx, caps, [z.copy() for z in zeros], [z.copy() for z in zeros], f16)
        p.load_payload(f.fileno(), nb)
        f.seek(0)
        ok_k = [np.zeros_like(z) for z in zeros]
        ok_v = [np.zeros_like(z) for z in zeros]
        S.load(1, f.read(), ctx, caps, ok_k, ok_v)
        for il in range(C.LAYERS):
            assert np.array_equal(_host(pk[il], f16), ok_k[il])
            assert np.array_equal(_host(pv[il], f16), ok_v[il])


def test_payload_streams_in_chunks():
    # 98 MB of payload rows: more than one 64 MB staging chunk each way
    ctx, n = 1024, 1000
    caps = [ctx] * C.LAYERS
    toks, lg, hd, kc, vc = C.state(9, ctx, n, caps, f16=True)
    s, _, _ = _session(ctx, caps, kc, vc, True, toks, lg, hd)
    with tempfile.TemporaryFile() as f:
        nb = s.save_payload(f)
        assert nb > (64 << 20)
        f.seek(0)
        pay = f.read()
        assert pay == S.save(1, ctx, toks, lg, hd, kc, vc, caps)
        f.seek(0)
        z = [np.zeros_like(a) for a in kc]
        r, rk, rv = _session(ctx, caps, z, [a.copy() for a in z], True)
        r.load_payload(f.fileno(), nb)
    ok_k = [np.zeros_like(a) for a in kc]
    ok_v = [np.zeros_like(a) for a in kc]
    S.load(1, pay, ctx, caps, ok_k, ok_v)
    for il in (0, 1, 22, 44):
        assert np.array_equal(_host(rk[il], True), ok_k[il])
        assert np.array_equal(_host(rv[il], True), ok_v[il])


@pytest.mark.parametrize("kind", [0, 1])
def test_loader_messages_match_oracle(kind):
    from sf37_b200.session import SessionError
    ctx, n = 6, 5
    caps = [ctx] * C.LAYERS
    toks, lg, hd, kc, vc = C.state(13, ctx, n, caps)
    s, _, _ = _session(ctx, caps, kc, vc, False, toks, lg, hd)
    if kind == 0:
        good = s.save_snapshot().numpy().tobytes()
    else:
        with tempfile.TemporaryFile() as f:
            s.save_payload(f)
            f.seek(0)
            good = f.read()
    for name, bad, lctx in C.corruptions(kind, good, ctx):
        z = [np.zeros((ctx, C.KV), np.float32) for _ in range(C.LAYERS)]
        with pytest.raises(S.LoadError) as want:
            S.load(kind, bad, lctx, caps, z, [a.copy() for a in z])
        r, _, _ = _session(lctx, caps, z, [a.copy() for a in z], False)
        with pytest.raises(SessionError) as got:
            if kind == 0:
                r.load_snapshot(bad)
            else:
                with tempfile.TemporaryFile() as f:
                    f.write(bad)
                    f.flush()
                    f.seek(0)
                    r.load_payload(f.fileno(), len(bad))
        assert str(got.value) == str(want.value), name


def test_loads_reference_payload_golden():
    g = np.load(GOLD)
    ctx, n = 3, 2
    toks, lg, hd, kc, vc = C.state(7, ctx, n, [ctx] * C.LAYERS, coarse=True)
    z = [np.zeros((ctx, C.KV), np.float32) for _ in range(C.LAYERS)]
    r, rk, rv = _session(ctx, [ctx] * C.LAYERS, z, [a.copy() for a in z], False)
    buf = g["payload"].tobytes()
    with tempfile.TemporaryFile() as f:
        f.write(buf)
        f.flush()
        f.seek(0)
        r.load_payload(f.fileno(), len(buf))
    assert r.n_tokens == n and np.array_equal(r.tokens[:n], toks)
    assert np.array_equal(r.logits, lg) and np.array_equal(r.hidden, hd)
    ok_k = [a.copy() for a in z]
    ok_v = [a.copy() for a in z]
    S.load(1, buf, ctx, [ctx] * C.LAYERS, ok_k, ok_v)
    for il in range(C.LAYERS):
        assert np.array_equal(rk[il].cpu().numpy(), ok_k[il])
        assert np.array_equal(rv[il].cpu().numpy(), ok_v[il])


def test_empty_session_roundtrip():
    # no tokens: header, row counts (all 0), logits and hidden only
    ctx = 16
    caps = [ctx] * C.LAYERS
    toks, lg, hd, kc, vc = C.state(17, ctx, 0, caps)
    s, _, _ = _session(ctx, caps, kc, vc, False, toks, lg, hd)
    snap = s.save_snapshot().numpy().tobytes()
    assert snap == S.save(0, ctx, toks, lg, hd, kc, vc, caps)
    with tempfile.TemporaryFile() as f:
        nb = s.save_payload(f)
        f.seek(0)
        pay = f.read()
        assert pay == S.save(1, ctx, toks, lg, hd, kc, vc, caps) and nb == len(pay)
        r, _, _ = _session(ctx, caps, kc, vc, False)
        f.seek(0)
        r.load_payload(f.fileno(), nb)
        assert r.n_tokens == 0 and np.array_equal(r.logits, lg)
    r.load_snapshot(snap)
    assert r.n_tokens == 0 and np.array_equal(r.hidden, hd)
