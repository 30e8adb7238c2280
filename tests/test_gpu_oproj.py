"""GPU: the Q8_0 o_proj matvec (sf37kv_oproj_q8_0 / sf37_cuda_matvec_q8_0)
against the oracle restatement of sf37_q8_0_matvec: activation codes and
scales bit for bit, outputs within float-accumulation bounds."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _check(out, w, x, out_dim):
    want = oracle.q8_0_matvec(w, x, out_dim)
    bound = 2e-6 * oracle.q8_0_abs_terms(w, x, out_dim) + 1e-30
    err = np.abs(out - want)
    assert np.all(err <= bound), (err.max(), (err / bound).max())


@pytest.mark.parametrize("n", [256, 8192, 12288])
def test_quantize_bit_exact(n):
    x = synth.normal(n, (n,)) * 3
    x[32:64] = 0
    x[100] = 1e30
    x[200:232] = 1e-30
    xq = torch.empty(n, dtype=torch.int8, device="cuda")
    xs = torch.empty(n // 32, dtype=torch.float32, device="cuda")
    xd = _dev(x)
    assert _lib.lib().sf37kv_q8_0_quantize(xd.data_ptr(), xq.data_ptr(), xs.data_ptr(), n, None) == 0
    wq, ws = oracle.q8_0_quantize(x)
    torch.cuda.synchronize()
    assert np.array_equal(xq.cpu().numpy(), wq)
    assert np.array_equal(xs.cpu().numpy(), ws)


@pytest.mark.parametrize("in_dim,out_dim", [(8192, 4096), (12288, 4096), (256, 8), (4096, 1000)])
def test_oproj_matches_oracle(in_dim, out_dim):
    w = synth.q8_0_weights(in_dim + out_dim, out_dim, in_dim)
    x = synth.normal(7, (in_dim,))
    out = torch.full((out_dim,), float("nan"), device="cuda")
    wd, xd = _dev(w), _dev(x)
    L = (_lib.OprojLayer * 1)(_lib.OprojLayer(wd.data_ptr(), xd.data_ptr(), out.data_ptr()))
    assert _lib.lib().sf37kv_oproj_q8_0(L, 1, in_dim, out_dim, None) == 0, _lib.last_error()
    torch.cuda.synchronize()
    _check(out.cpu().numpy(), w, x, out_dim)


def test_oproj_batched_layers_and_dropin():
    in_dim, out_dim, n = 8192, 512, 6
    ws = [synth.q8_0_weights(50 + i, out_dim, in_dim) for i in range(n)]
    xs = [synth.normal(60 + i, (in_dim,)) * (i + 1) for i in range(n)]
    wd = [_dev(w) for w in ws]
    xd = [_dev(x) for x in xs]
    outs = [torch.empty(out_dim, device="cuda") for _ in range(n)]
    L = (_lib.OprojLayer * n)(*[_lib.OprojLayer(wd[i].data_ptr(), xd[i].data_ptr(), outs[i].data_ptr())
                                for i in range(n)])
    assert _lib.lib().sf37kv_oproj_q8_0(L, n, in_dim, out_dim, None) == 0
    torch.cuda.synchronize()
    for i in range(n):
        _check(outs[i].cpu().numpy(), ws[i], xs[i], out_dim)
    # the reference-API entry point on tensor handles
    o = torch.empty(out_dim, device="cuda")
    T = _lib.Tensor
    assert _lib.lib().sf37_cuda_matvec_q8_0(ctypes.byref(T(o.data_ptr(), o.numel() * 4)),
                                            ctypes.byref(T(wd[0].data_ptr(), wd[0].numel())), in_dim, out_dim,
                                            ctypes.byref(T(xd[0].data_ptr(), xd[0].numel() * 4))) == 1
    torch.cuda.synchronize()
    assert torch.equal(o, outs[0])
    # too-small tensors -> 0 (sf37_cuda.cu:3714-3716)
    assert _lib.lib().sf37_cuda_matvec_q8_0(ctypes.byref(T(o.data_ptr(), 4)),
                                            ctypes.byref(T(wd[0].data_ptr(), wd[0].numel())), in_dim, out_dim,
                                            ctypes.byref(T(xd[0].data_ptr(), xd[0].numel() * 4))) == 0


def test_oproj_rejects_unsupported():
    w = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    x = torch.zeros(64, device="cuda")
    o = torch.zeros(4, device="cuda")
    L = (_lib.OprojLayer * 1)(_lib.OprojLayer(w.data_ptr(), x.data_ptr(), o.data_ptr()))
    assert _lib.lib().sf37kv_oproj_q8_0(L, 1, 64, 4, None) == 4  # in_dim % 256
    L[0].x = x.data_ptr() + 4
    assert _lib.lib().sf37kv_oproj_q8_0(L, 1, 256, 4, None) == 1  # alignment
