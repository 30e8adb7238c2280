"""GPU parity against the reference's OWN CUDA kernels (sf37_cuda.cu built
for sm_100a from the reference sources, oracle/_ref/libsf37ref_cuda.so) on
identical device inputs: append bit-exact, attention within tolerance.  This
covers ring wrap, cap clamp and split-K sizes the reference CPU code cannot
express."""
import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import kv, synth
from tests.gpu_util import dev, host
from tests.helpers import F32_TOL, assert_close

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.ref_cuda_available(), reason="reference CUDA lib not built")]


def _rt(t):
    return oracle.ref_tensor(t.data_ptr(), t.numel() * t.element_size())


@pytest.mark.parametrize("pos,cap,sliding,qh", [(2048, 2049, 0, 64), (32768, 32769, 0, 64),
                                                (70000, 520, 1, 96), (5000, 1024, 1, 64),
                                                (100, 8192, 1, 96), (1200, 1000, 0, 64)])
def test_decode_at_vs_reference_cuda(pos, cap, sliding, qh):
    R = oracle.ref_cuda()
    kd = 1024
    k = dev(synth.normal(61 + pos, (cap, kd)))
    v = dev(synth.normal(62 + pos, (cap, kd)))
    q = dev(synth.normal(63, (qh, 128)))
    g = dev(synth.normal(64, (qh,)))
    ours = torch.empty(qh, 128, device="cuda")
    theirs = torch.empty(qh, 128, device="cuda")
    assert kv.attention_decode_heads_at(ours, q, k, v, g, pos, cap, qh, 8, 128, sliding, 512)
    torch.cuda.synchronize()
    assert R.sf37_cuda_attention_decode_heads_at(_rt(theirs), _rt(q), _rt(k), _rt(v), _rt(g), pos, cap,
                                                 qh, 8, 128, sliding, 512)
    assert R.sf37_cuda_synchronize()
    assert_close(host(ours), host(theirs), atol=F32_TOL, rtol=1e-4)


def test_append_and_prefill_vs_reference_cuda():
    R = oracle.ref_cuda()
    n_tok, pos0, cap, qh, kvh = 40, 500, 512, 64, 8
    kd, qd = kvh * 128, qh * 128
    kn, vn = dev(synth.normal(71, (n_tok, kd))), dev(synth.normal(72, (n_tok, kd)))
    base_k, base_v = synth.normal(73, (cap, kd)), synth.normal(74, (cap, kd))
    ka, va, kb, vb = dev(base_k), dev(base_v), dev(base_k), dev(base_v)
    q = dev(synth.normal(75, (n_tok, qd)))
    g = dev(synth.normal(76, (n_tok, qh)))
    assert kv.store_kv_cache_batch(ka, va, kn, vn, pos0, n_tok, cap, kd)
    torch.cuda.synchronize()
    assert R.sf37_cuda_store_kv_cache_batch(_rt(kb), _rt(vb), _rt(kn), _rt(vn), pos0, n_tok, cap, kd)
    assert R.sf37_cuda_synchronize()
    assert torch.equal(ka, kb) and torch.equal(va, vb)
    ours = torch.empty(n_tok, qd, device="cuda")
    theirs = torch.empty(n_tok, qd, device="cuda")
    assert kv.attention_prefill_heads(ours, q, ka, va, g, pos0, n_tok, cap, qh, kvh, 128, 1, 472)
    torch.cuda.synchronize()
    assert R.sf37_cuda_attention_prefill_heads(_rt(theirs), _rt(q), _rt(kb), _rt(vb), _rt(g), pos0, n_tok,
                                               cap, qh, kvh, 128, 1, 472)
    assert R.sf37_cuda_synchronize()
    assert_close(host(ours), host(theirs), atol=F32_TOL, rtol=1e-4)
