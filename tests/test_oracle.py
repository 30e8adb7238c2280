"""CPU: the oracle restatement pinned against the reference's own code
(golden fixtures from oracle/_ref, and the live reference library when it is
present) and against the reference's own self-tests."""
import os

import numpy as np
import pytest

import oracle
from sf37_b200 import synth
from tests.helpers import assert_close

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _g(name):
    return np.load(os.path.join(GOLD, name))


def test_payload_encode_matches_reference_golden():
    g = _g("payload_rows.npz")
    enc = oracle.payload_encode_rows(g["rows"], 64, variant=1)
    assert np.array_equal(enc, g["enc"])
    assert np.array_equal(oracle.payload_decode_rows(g["enc"], 1024), g["dec"])


def test_payload_literal_variant_differs_on_ties():
    # The source-literal IEEE form is not what the compiled reference emits.
    g = _g("payload_rows.npz")
    enc0 = oracle.payload_encode_rows(g["rows"], 64, variant=0)
    assert not np.array_equal(enc0, g["enc"])


def test_payload_reference_self_test():
    # sf37.c:6676-6726: row size, pattern roundtrip < 0.02, zero row exact.
    assert oracle.payload_row_bytes(1024, 64) == 16 * 4 + 1024
    pat = ((np.arange(1024) % 97).astype(np.int32) - 48).astype(np.float32) / np.float32(13.0)
    dec = oracle.payload_decode_rows(oracle.payload_encode_rows(pat[None]), 1024)[0]
    assert np.abs(dec - pat).max() < 0.02
    z = np.zeros((1, 1024), np.float32)
    assert np.all(oracle.payload_decode_rows(oracle.payload_encode_rows(z), 1024) == 0)


def test_payload_nonfinite_inputs():
    x = synth.normal(7, (1, 1024))
    x[0, 3] = np.inf
    x[0, 70] = np.nan
    enc = oracle.payload_encode_rows(x)
    q = enc[0, 64:].view(np.int8)
    assert q[3] == 0 and q[70] == 0


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
@pytest.mark.parametrize("scale", [1.0, 3.0, 1e-3, 250.0])
def test_payload_encode_matches_live_reference(scale):
    x = synth.normal(11 + int(scale * 10), (3000, 1024)) * np.float32(scale)
    assert np.array_equal(oracle.payload_encode_rows(x), oracle.ref_payload_encode_rows(x))


def test_cfg1_attention_matches_reference_golden():
    g = _g("cfg1_decode.npz")
    k, v, k_new, v_new, q, gate = synth.cfg1_inputs(0)
    cap = 4096  # ring larger than the live rows: identical to the linear cache
    kc = np.zeros((cap, 1024), np.float32)
    vc = np.zeros((cap, 1024), np.float32)
    oracle.store_kv_rows(kc, vc, k.astype(np.float32), v.astype(np.float32), 0, 2048, cap, 1024)
    oracle.store_kv_rows(kc, vc, k_new[None], v_new[None], 2048, 1, cap, 1024)
    out = oracle.attention_decode_at(q, kc, vc, None, 2048, cap, 64, 8, 128)
    assert_close(out, g["out_nogate"], atol=1e-6, rtol=1e-5, what="cfg1 no gate")
    out = oracle.attention_decode_at(q, kc, vc, gate, 2048, cap, 64, 8, 128)
    assert_close(out, g["out_gate"], atol=1e-6, rtol=1e-5, what="cfg1 gate")


def test_sliding_attention_matches_reference_golden():
    g = _g("sliding_decode.npz")
    ks = synth.normal(201, (600, 1024))
    vs = synth.normal(202, (600, 1024))
    qs = synth.normal(203, (96, 128))
    gs = synth.normal(204, (96,))
    # the reference's linear cache of 600 rows = a ring of cap 600 at pos 599
    out = oracle.attention_decode_at(qs, ks, vs, gs, 599, 600, 96, 8, 128, sliding=1, window=512)
    assert_close(out, g["out"], atol=1e-6, rtol=1e-5, what="sliding")
    out_n = oracle.attention_decode_n(qs, ks, vs, gs, 600, 600, 96, 8, 128, sliding=1, window=512)
    assert_close(out_n, g["out"], atol=1e-6, rtol=1e-5, what="sliding n_cache form")


def test_ring_append_equals_reference_linear_push():
    # kv_cache_push memmoves when full (sf37.c:2054-2064); the ring keeps the
    # same live rows at slot pos % cap.
    g = _g("kv_push.npz")
    kp = synth.normal(301, (6, 1024))
    vp = synth.normal(302, (6, 1024))
    kc = np.zeros((4, 1024), np.float32)
    vc = np.zeros((4, 1024), np.float32)
    oracle.store_kv_rows(kc, vc, kp, vp, 0, 6, 4, 1024)
    n = int(g["n"])
    for i in range(n):
        pos = 6 - n + i
        assert np.array_equal(kc[pos % 4], g["k"][i])
        assert np.array_equal(vc[pos % 4], g["v"][i])


def test_f16_conversion_is_ieee_rne():
    x = np.concatenate([synth.normal(5, (200000,)) * np.float32(300),
                        synth.normal(6, (50000,)) * np.float32(1e-5),
                        np.array([65504, 65519, 65520, 1e9, -1e9, 6e-8, 2.98e-8, -0.0, 0.0],
                                 np.float32)])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16_bits(x), want)
    h = np.arange(65536, dtype=np.uint16)
    f = oracle.f16_bits_to_f32(h)
    ref = h.view(np.float16).astype(np.float32)
    assert np.all((f == ref) | (np.isnan(f) & np.isnan(ref)))


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
@pytest.mark.parametrize("n,sliding,q_heads", [(1, 0, 64), (17, 0, 64), (700, 1, 64), (513, 1, 96)])
def test_attention_matches_live_reference(n, sliding, q_heads):
    k = synth.normal(400 + n, (n, 1024))
    v = synth.normal(500 + n, (n, 1024))
    q = synth.normal(600 + n, (q_heads, 128))
    gate = synth.normal(700 + n, (q_heads,))
    want = oracle.ref_attention_decode(q, k, v, n, n, q_heads, sliding, gate)
    got = oracle.attention_decode_at(q, k, v, gate, n - 1, n, q_heads, 8, 128, sliding, 512)
    assert_close(got, want, atol=1e-6, rtol=1e-5)


# q/k head preparation: fast-math in the reference build (FMA contraction,
# reassociated products) moves results by about one ulp, so the restatement
# is pinned within 2 ulp-scale bounds rather than bit for bit.
QK_ATOL, QK_RTOL = 2e-6, 1e-6


def test_qk_prep_matches_reference_golden():
    g = _g("qk_prep.npz")
    for i, p in enumerate(g["pos"]):
        got_f = oracle.qk_prep(g["x"][i], g["w"], 64, 5e6, True, int(p))
        got_s = oracle.qk_prep(g["x"][i], g["w"], 128, 1e4, False, int(p))
        np.testing.assert_allclose(got_f, g["full"][i], rtol=QK_RTOL, atol=QK_ATOL)
        np.testing.assert_allclose(got_s, g["sliding"][i], rtol=QK_RTOL, atol=QK_ATOL)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
def test_qk_prep_matches_live_reference():
    rng = np.random.default_rng(5)
    w = ((rng.standard_normal(128) * 0.3).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    for p in rng.integers(0, 262144, 40):
        x = (rng.standard_normal((16, 128)) * 4).astype(np.float32)
        for rot, th, ll in ((64, 5e6, 1), (128, 1e4, 0), (32, 1e4, 0)):
            np.testing.assert_allclose(oracle.qk_prep(x, w, rot, th, ll, int(p)),
                                       oracle.ref_qk_prep(x, w, rot, th, ll, int(p)), rtol=QK_RTOL, atol=QK_ATOL)
    # zero head: scale = 1/sqrt(eps) times zero stays zero
    z = np.zeros((1, 128), np.float32)
    assert not np.any(oracle.qk_prep(z, w, 64, 5e6, 1, 9))


# ---- Q8_0 o_proj matvec ----
def _tie_only(a_q, b_q, x, xs):
    """Codes may differ only where x / scale sits on a .5 tie: the reference
    build vectorizes iscale * x into a CPU-specific reciprocal estimate."""
    d = np.nonzero(a_q != b_q)[0]
    assert np.all(np.abs(a_q[d].astype(int) - b_q[d].astype(int)) == 1)
    for i in d:
        t = float(x[i]) / float(xs[i // 32])
        assert abs(abs(t - np.trunc(t)) - 0.5) < 1e-5 * max(1.0, abs(t)), (i, t)
    return d.size


def test_q8_0_matches_reference_golden():
    g = _g("q8_0.npz")
    x = synth.normal(30, (8192,)) * 2
    x[64:96] = 0
    w = synth.q8_0_weights(31, 16, 8192)
    xq, xs = oracle.q8_0_quantize(x)
    assert np.array_equal(xs, g["xs"])
    _tie_only(xq, g["xq"], x, xs)
    assert not np.any(xq[64:96]) and xs[2] == 0
    # the reference build reassociates the float accumulation: ulp-scale
    out = oracle.q8_0_matvec(w, x, 16)
    scale = oracle.q8_0_abs_terms(w, x, 16)
    assert np.all(np.abs(out - g["out"]) <= 1e-6 * scale + 1e-7)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
def test_q8_0_matches_live_reference():
    rng = np.random.default_rng(8)
    ties = 0
    for t in range(20):
        x = (rng.standard_normal(4096) * rng.choice([1e-3, 1.0, 40.0])).astype(np.float32)
        xq, xs = oracle.q8_0_quantize(x)
        rq, rs = oracle.ref_q8_0_quantize(x)
        assert np.array_equal(xs, rs)
        ties += _tie_only(xq, rq, x, xs)
        w = synth.q8_0_weights(100 + t, 32, 4096)
        out = oracle.q8_0_matvec(w, x, 32)
        ref = oracle.ref_q8_0_matvec(w, x, 32)
        assert np.all(np.abs(out - ref) <= 1e-6 * oracle.q8_0_abs_terms(w, x, 32) + 1e-30)
    assert ties < 20  # ties are rare (about 1 in 10^5 codes)
