"""GPU parity: chunked-prefill attention (sf37_cuda.cu:3163-3317) vs the
oracle (cpu_attention_prefill_ref, tests/test_sf37_cuda_ops.cu:859-905)."""
import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import kv, synth
from tests.gpu_util import dev, f16_cache, host
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


def test_reference_prefill_case():
    # tests/test_sf37_cuda_ops.cu:1112-1150: n_tok 3, pos0 2, cap 8, 8/2 heads, tol 6e-5
    n_tok, pos0, qh, kvh, hd, cap = 3, 2, 8, 2, 128, 8
    qd, kd = qh * hd, kvh * hd
    q = (((np.arange(n_tok * qd) % 37) - 18) * 0.006).astype(np.float32).reshape(n_tok, qd)
    k = (((np.arange(n_tok * kd) % 31) - 15) * 0.005).astype(np.float32).reshape(n_tok, kd)
    v = (((np.arange(n_tok * kd) % 29) - 14) * 0.007).astype(np.float32).reshape(n_tok, kd)
    g = (((np.arange(n_tok * qh) % 11) - 5) * 0.09).astype(np.float32).reshape(n_tok, qh)
    kc = (((np.arange(cap * kd) % 23) - 11) * 0.004).astype(np.float32).reshape(cap, kd)
    vc = (((np.arange(cap * kd) % 19) - 9) * 0.008).astype(np.float32).reshape(cap, kd)
    dkc, dvc = dev(kc), dev(vc)
    out = torch.empty(n_tok, qd, device="cuda")
    assert kv.store_kv_cache_batch(dkc, dvc, dev(k), dev(v), pos0, n_tok, cap, kd)
    assert kv.attention_prefill_heads(out, dev(q), dkc, dvc, dev(g), pos0, n_tok, cap, qh, kvh, hd, 0, 512)
    oracle.store_kv_rows(kc, vc, k, v, pos0, n_tok, cap, kd)
    want = oracle.attention_prefill(q, kc, vc, g, pos0, n_tok, cap, qh, kvh, hd)
    assert_close(host(out).reshape(n_tok, qh, hd), want, atol=6e-5, rtol=0)


@pytest.mark.parametrize("qtype", ["f32", "bf16"])
@pytest.mark.parametrize("pos0,n_tok,cap,sliding", [(0, 64, 64, 0), (300, 130, 1024, 0),
                                                    (1000, 200, 768, 1), (5, 1, 16, 0)])
def test_native_prefill_f16(qtype, pos0, n_tok, cap, sliding):
    qh, kvh, hd = 64, 8, 128
    kd = kvh * hd
    kc, kref = f16_cache(synth.normal(11 + pos0, (cap, kd)))
    vc, vref = f16_cache(synth.normal(12 + pos0, (cap, kd)))
    qf = synth.normal(13 + pos0, (n_tok, qh, hd))
    tq = dev(qf)
    if qtype == "bf16":
        tq = tq.to(torch.bfloat16)
        qf = tq.float().cpu().numpy()
    g = synth.normal(14, (n_tok, qh))
    out = torch.empty(n_tok, qh, hd, device="cuda")
    kv.prefill(kc, vc, cap, tq, dev(g), out, pos0, n_tok, qh, kvh, hd, kv.F16, sliding=sliding)
    want = oracle.attention_prefill(qf, kref, vref, g, pos0, n_tok, cap, qh, kvh, hd, sliding, 512)
    assert_close(host(out), want)


@pytest.mark.parametrize("G,pos0,n_tok,cap,sliding", [(8, 2000, 300, 2400, 1), (8, 3000, 1000, 4096, 0),
                                                      (12, 700, 257, 1024, 1), (4, 0, 33, 64, 0),
                                                      (16, 90, 70, 256, 0)])
def test_tensor_core_prefill_bf16(G, pos0, n_tok, cap, sliding):
    kvh = 4 if G > 8 else 8
    qh, hd = G * kvh, 128
    kd = kvh * hd
    kc, kref = f16_cache(synth.normal(51 + G, (cap, kd)))
    vc, vref = f16_cache(synth.normal(52 + G, (cap, kd)))
    tq = dev(synth.normal(53, (n_tok, qh, hd))).to(torch.bfloat16)
    qf = tq.float().cpu().numpy()
    g = synth.normal(54, (n_tok, qh))
    out = torch.empty(n_tok, qh, hd, device="cuda")
    kv.prefill(kc, vc, cap, tq, dev(g), out, pos0, n_tok, qh, kvh, hd, kv.F16, sliding=sliding)
    got = host(out)
    from sf37_b200 import _lib
    assert _lib.lib().sf37kv_device_error(1) == 0, "a bounded wait in the prefill kernel gave up"
    # all tokens for small chunks; a sampled prefix + suffix otherwise
    spans = [(0, n_tok)] if n_tok <= 300 else [(0, 40), (n_tok - 40, n_tok)]
    for a, b in spans:
        want = oracle.attention_prefill(qf, kref, vref, g, pos0, n_tok, cap, qh, kvh, hd, sliding, 512,
                                        t0=a, t1=b)
        assert_close(got[a:b], want[a:b], what=f"tokens {a}..{b}")


@pytest.mark.parametrize("G,pos0,n_tok,cap,sliding", [(8, 0, 64, 64, 0), (8, 300, 130, 1024, 0),
                                                      (8, 1000, 200, 768, 1), (4, 5, 1, 16, 0),
                                                      (8, 2000, 257, 2400, 1), (4, 700, 100, 750, 0),
                                                      (8, 90, 70, 128, 0)])
def test_dropin_prefill_f32_tensor_cores(G, pos0, n_tok, cap, sliding):
    # fp32 caches and fp32 q (the engine's sf37_cuda_attention_prefill_heads
    # call, sf37.c:5919): the bf16 hi/lo tensor-core kernel, held to the
    # reference tests' fp32 tolerance; (700, 100, 750) and (90, 70, 128) wrap
    # the ring inside the chunk.
    kvh = 8 if G == 8 else 4
    qh, hd = G * kvh, 128
    kd = kvh * hd
    k = synth.normal(61 + G + pos0, (cap, kd))
    v = synth.normal(62 + G + pos0, (cap, kd))
    q = synth.normal(63 + pos0, (n_tok, qh * hd))
    g = synth.normal(64, (n_tok, qh))
    out = torch.empty(n_tok, qh * hd, device="cuda")
    assert kv.attention_prefill_heads(out, dev(q), dev(k), dev(v), dev(g), pos0, n_tok, cap, qh, kvh, hd,
                                      sliding, 512)
    want = oracle.attention_prefill(q, k, v, g, pos0, n_tok, cap, qh, kvh, hd, sliding, 512)
    assert_close(host(out).reshape(n_tok, qh, hd), want, atol=6e-5, rtol=1e-4, what=f"G={G}")


def test_native_prefill_f32_cache_bf16_q():
    # f32 cache + bf16 queries through sf37kv_prefill: q widened, then the
    # fp32 tensor-core kernel
    qh, kvh, hd, cap, pos0, n_tok = 64, 8, 128, 4096, 3000, 300
    kd = kvh * hd
    k = synth.normal(71, (cap, kd))
    v = synth.normal(72, (cap, kd))
    tq = dev(synth.normal(73, (n_tok, qh, hd))).to(torch.bfloat16)
    qf = tq.float().cpu().numpy()
    g = synth.normal(74, (n_tok, qh))
    out = torch.empty(n_tok, qh, hd, device="cuda")
    kv.prefill(dev(k), dev(v), cap, tq, dev(g), out, pos0, n_tok, qh, kvh, hd, kv.F32)
    want = oracle.attention_prefill(qf, k, v, g, pos0, n_tok, cap, qh, kvh, hd)
    assert_close(host(out), want, atol=6e-5, rtol=1e-4)
