"""GPU parity: decode attention through the C ABI vs the oracle (and the
reference's own golden outputs), f32 drop-in and f16 native paths."""
import os

import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import kv, synth
from tests.gpu_util import dev, f16_cache, host
from tests.helpers import F32_TOL, assert_close

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _pattern_case(q_heads, kv_heads, hd, cap):
    # integer-pattern inputs of the reference test (tests/test_sf37_cuda_ops.cu:310-320)
    q = (((np.arange(q_heads * hd) % 23) - 11) * 0.013).astype(np.float32).reshape(q_heads, hd)
    n = cap * kv_heads * hd
    k = (((np.arange(n) % 29) - 14) * 0.009).astype(np.float32).reshape(cap, kv_heads * hd)
    v = (((np.arange(n) % 31) - 15) * 0.011).astype(np.float32).reshape(cap, kv_heads * hd)
    g = ((np.arange(q_heads) - 4) * 0.17).astype(np.float32)
    return q, k, v, g


def test_reference_tiny_case():
    # tests/test_sf37_cuda_ops.cu:274-300: 4 Q / 2 KV heads, d 8, cap 4, n 3, tol 2e-5
    hd, qh, kvh, cap = 8, 4, 2, 4
    q = (((np.arange(qh * hd) % 11) - 5) * 0.08).astype(np.float32).reshape(qh, hd)
    k = (((np.arange(cap * kvh * hd) % 13) - 6) * 0.05).astype(np.float32).reshape(cap, kvh * hd)
    v = (((np.arange(cap * kvh * hd) % 7) - 3) * 0.09).astype(np.float32).reshape(cap, kvh * hd)
    g = ((np.arange(qh) - 2) * 0.4).astype(np.float32)
    out = torch.empty(qh, hd, device="cuda")
    assert kv.attention_decode_heads(out, dev(q), dev(k), dev(v), dev(g), 3, cap, qh, kvh, hd, 0, 0)
    want = oracle.attention_decode_n(q, k, v, g, 3, cap, qh, kvh, hd)
    assert_close(host(out), want, atol=2e-5, rtol=0)


@pytest.mark.parametrize("n", [1, 2, 17, 513])
def test_reference_d128_cases(n):
    # tests/test_sf37_cuda_ops.cu:304-336: 8 Q / 2 KV heads, cap 520, sliding at 513, tol 5e-5
    q, k, v, g = _pattern_case(8, 2, 128, 520)
    sliding = int(n == 513)
    out = torch.empty(8, 128, device="cuda")
    assert kv.attention_decode_heads(out, dev(q), dev(k), dev(v), dev(g), n, 520, 8, 2, 128, sliding, 512)
    want = oracle.attention_decode_n(q, k, v, g, n, 520, 8, 2, 128, sliding, 512)
    assert_close(host(out), want, atol=5e-5, rtol=0)


@pytest.mark.parametrize("G", [1, 2, 4, 8, 12, 16, 3, 5])
@pytest.mark.parametrize("rows,cap,pos,sliding", [(0, 64, 0, 0), (1023, 1500, 1022, 0),
                                                  (1025, 1025, 3000, 0), (4097, 4097, 4096, 0),
                                                  (0, 700, 2000, 1), (0, 512, 70000, 1)])
def test_dropin_decode_at_f32(G, rows, cap, pos, sliding):
    kvh = 2 if G > 4 else 4
    qh = G * kvh
    kd = kvh * 128
    k = synth.normal(31 + G + pos, (cap, kd))
    v = synth.normal(32 + G + pos, (cap, kd))
    q = synth.normal(33 + G, (qh, 128))
    g = synth.normal(34 + G, (qh,))
    out = torch.empty(qh, 128, device="cuda")
    assert kv.attention_decode_heads_at(out, dev(q), dev(k), dev(v), dev(g), pos, cap, qh, kvh, 128,
                                        sliding, 512)
    want = oracle.attention_decode_at(q, k, v, g, pos, cap, qh, kvh, 128, sliding, 512)
    assert_close(host(out), want, atol=F32_TOL, rtol=1e-4, what=f"G={G}")


def test_cfg1_f16_vs_reference_golden():
    gold = np.load(os.path.join(GOLD, "cfg1_decode.npz"))
    k, v, k_new, v_new, q, gate = synth.cfg1_inputs(0)
    cap = 2049
    kc, _ = f16_cache(np.vstack([k.astype(np.float32), np.zeros((1, 1024), np.float32)]))
    vc, _ = f16_cache(np.vstack([v.astype(np.float32), np.zeros((1, 1024), np.float32)]))
    # The golden reference cache holds the fp32 new row; the f16 cache holds
    # its RNE image, so compare against the oracle on those bits too.
    out = torch.empty(64, 128, device="cuda")
    layer = dict(k_cache=kc, v_cache=vc, cap=cap, pos=2048, q=dev(q), gate=dev(gate), out=out,
                 k_new=dev(k_new), v_new=dev(v_new))
    kv.decode([layer], 64, 8, 128, kv.F16)
    got = host(out)
    assert_close(got, gold["out_gate"], what="cfg1 vs reference (fp32 new row)")
    kf = oracle.f16_bits_to_f32(kc.cpu().view(torch.int16).numpy().view(np.uint16))
    vf = oracle.f16_bits_to_f32(vc.cpu().view(torch.int16).numpy().view(np.uint16))
    want = oracle.attention_decode_at(q, kf, vf, gate, 2048, cap, 64, 8, 128)
    assert_close(got, want, what="cfg1 vs oracle on f16 bits")


@pytest.mark.parametrize("G", [8, 12, 4, 16, 1])
def test_native_f16_multilayer_mixed(G):
    kvh = 8 if G <= 8 else 4
    qh = G * kvh
    kd = kvh * 128
    specs = [(5000, 5000, 4999, 0), (512, 512, 9000, 1), (1024, 1536, 777, 1), (64, 64, 31, 0),
             (3000, 2048, 2500, 0), (8192, 8192, 100000, 1)]
    layers, want = [], []
    for i, (_, cap, pos, sliding) in enumerate(specs):
        kf = synth.normal(1000 + i, (cap, kd))
        vf = synth.normal(2000 + i, (cap, kd))
        kc, kref = f16_cache(kf)
        vc, vref = f16_cache(vf)
        q = synth.normal(3000 + i, (qh, 128))
        g = synth.normal(4000 + i, (qh,))
        kn = synth.normal(5000 + i, (kd,))
        vn = synth.normal(6000 + i, (kd,))
        out = torch.empty(qh, 128, device="cuda")
        layers.append(dict(k_cache=kc, v_cache=vc, cap=cap, sliding=sliding, window=512, pos=pos,
                           q=dev(q), gate=dev(g), out=out, k_new=dev(kn), v_new=dev(vn)))
        hk = oracle.f32_to_f16_bits(kf)
        hv = oracle.f32_to_f16_bits(vf)
        oracle.store_kv_rows(hk, hv, kn[None], vn[None], pos, 1, cap, kd)
        want.append(oracle.attention_decode_at(q, oracle.f16_bits_to_f32(hk), oracle.f16_bits_to_f32(hv),
                                               g, pos, cap, qh, kvh, 128, sliding, 512))
    kv.decode(layers, qh, kvh, 128, kv.F16)
    for i, L in enumerate(layers):
        assert_close(host(L["out"]), want[i], what=f"layer {i}")


def test_f16_repeated_calls_reuse_scratch():
    # Split-K counters reset themselves: calling twice gives the same result.
    kd, cap = 1024, 6000
    kc, kref = f16_cache(synth.normal(71, (cap, kd)))
    vc, vref = f16_cache(synth.normal(72, (cap, kd)))
    q = synth.normal(73, (64, 128))
    outs = []
    for _ in range(3):
        out = torch.empty(64, 128, device="cuda")
        kv.decode([dict(k_cache=kc, v_cache=vc, cap=cap, pos=cap - 1, q=dev(q), out=out)], 64, 8, 128,
                  kv.F16)
        outs.append(host(out))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    want = oracle.attention_decode_at(q, kref, vref, None, cap - 1, cap, 64, 8, 128)
    assert_close(outs[0], want)


def test_gqa_single_token():
    v = synth.normal(81, (8 * 128,))
    g = synth.normal(82, (64,))
    out = torch.empty(64, 128, device="cuda")
    assert kv.gqa_single_token_heads(out, dev(v), dev(g), 64, 8, 128)
    want = v.reshape(8, 1, 128).repeat(8, axis=1).reshape(64, 128) * (1 / (1 + np.exp(-g)))[:, None]
    assert_close(host(out), want, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("f16", [True, False])
def test_back_to_back_steps_on_one_cache(f16):
    # Consecutive decode launches on the same stream, each appending the row
    # the next one reads (the programmatic-dependent-launch case: a kernel may
    # start before the previous one finished, and must not read early).
    cap, pos0, steps = 3000, 2500, 6
    k = synth.normal(71, (cap, 1024))
    v = synth.normal(72, (cap, 1024))
    kn = synth.normal(73, (steps, 1024))
    vn = synth.normal(74, (steps, 1024))
    qs = synth.normal(75, (steps, 64, 128))
    if f16:
        kb, vb = oracle.f32_to_f16_bits(k), oracle.f32_to_f16_bits(v)
        kd = torch.from_numpy(kb.view(np.float16)).cuda()
        vd = torch.from_numpy(vb.view(np.float16)).cuda()
        ke, ve = kb.copy(), vb.copy()
    else:
        kd, vd = dev(k), dev(v)
        ke, ve = k.copy(), v.copy()
    outs = [torch.empty(64, 128, device="cuda") for _ in range(steps)]
    qd, knd, vnd = dev(qs), dev(kn), dev(vn)
    for s in range(steps):
        kv.decode([dict(k_cache=kd, v_cache=vd, cap=cap, pos=pos0 + s, q=qd[s], out=outs[s],
                        k_new=knd[s], v_new=vnd[s])], 64, 8, 128, kv.F16 if f16 else kv.F32)
    torch.cuda.synchronize()
    for s in range(steps):
        oracle.store_kv_rows(ke, ve, kn[s:s + 1], vn[s:s + 1], pos0 + s, 1, cap, 1024)
        want = oracle.attention_decode_at(qs[s], ke, ve, None, pos0 + s, cap, 64, 8, 128)
        assert_close(host(outs[s]), want, what=f"step {s}")
