"""GPU: the allocation-free decode entry point (sf37kv_decode_noalloc).

Callers that cannot call cudaMalloc while decoding (a memory pool that owns
the whole device, allocations frozen after start-up) use this entry point;
its split-K scratch is a fixed device array inside the library.  These tests
call it through the C ABI and check it against the regular entry point
(sf37kv_decode) on the same inputs, twice in a row, since every call reuses
the same array.  The file is named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

from sf37_b200 import _lib, kv, synth
from tests.helpers import ATOL, RTOL, F32_TOL, assert_close

pytestmark = pytest.mark.gpu


def _layers(dtype, specs, qh, kvh, seed):
    kd = kvh * 128
    tdt = torch.float16 if dtype == kv.F16 else torch.float32
    out = []
    for i, (cap, pos, sliding) in enumerate(specs):
        g = torch.Generator(device="cuda")
        g.manual_seed(seed + i)
        kc = torch.randn(cap, kd, device="cuda", generator=g).to(tdt)
        vc = torch.randn(cap, kd, device="cuda", generator=g).to(tdt)
        out.append(dict(k_cache=kc, v_cache=vc, cap=cap, pos=pos, sliding=sliding, window=512,
                        q=torch.randn(qh, 128, device="cuda", generator=g),
                        gate=torch.randn(qh, device="cuda", generator=g)))
    return out


def _run(entry, layers, qh, kvh, dtype):
    outs = []
    for L in layers:
        L["out"] = torch.full((qh, 128), float("nan"), device="cuda")
        outs.append(L["out"])
    arr = kv.decode_layers_desc(layers)
    rc = getattr(_lib.lib(), entry)(arr, len(arr), qh, kvh, 128, dtype, None)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs]


CASES = [
    (kv.F16, 64, 8, [(2049, 2048, 0)]),
    (kv.F16, 64, 8, [(32769, 32768, 0), (512, 70000, 1), (9000, 8999, 0), (4096, 5000, 1)]),
    (kv.F16, 48, 4, [(20000, 19999, 0), (600, 1000, 1)]),       # group 12
    (kv.F32, 64, 8, [(6000, 5999, 0), (512, 3000, 1)]),
]


@pytest.mark.parametrize("dtype,qh,kvh,specs", CASES)
def test_noalloc_matches_regular_entry_twice(dtype, qh, kvh, specs):
    layers = _layers(dtype, specs, qh, kvh, seed=77)
    want = _run("sf37kv_decode", layers, qh, kvh, dtype)
    tol = dict(atol=ATOL, rtol=RTOL) if dtype == kv.F16 else dict(atol=F32_TOL, rtol=1e-4)
    for call in range(2):
        got = _run("sf37kv_decode_noalloc", layers, qh, kvh, dtype)
        for i, (g, w) in enumerate(zip(got, want)):
            assert np.isfinite(g).all(), f"call {call} layer {i}: output not written"
            assert_close(g, w, what=f"call {call} layer {i}", **tol)


def test_noalloc_many_layers_exercises_capacity():
    # 48 layers x 32K rows: the split plan must be coarsened to fit the fixed
    # partial buffer; results still match.
    layers = _layers(kv.F16, [(8192, 8191, 0)] * 48, 64, 8, seed=5)
    want = _run("sf37kv_decode", layers, 64, 8, kv.F16)
    for _ in range(2):
        got = _run("sf37kv_decode_noalloc", layers, 64, 8, kv.F16)
        for g, w in zip(got, want):
            assert_close(g, w)


def test_noalloc_rejects_oversize_and_unsupported():
    L = _lib.lib()
    arr = (_lib.DecodeLayer * 65)()
    assert L.sf37kv_decode_noalloc(arr, 65, 64, 8, 128, kv.F16, None) == 1
    assert "maximum" in _lib.last_error()
    arr1 = (_lib.DecodeLayer * 1)()
    arr1[0].cache.cap = 4
    arr1[0].cache.k_cache = arr1[0].cache.v_cache = arr1[0].q = arr1[0].out = 256
    assert L.sf37kv_decode_noalloc(arr1, 1, 8, 2, 64, kv.F16, None) == 4
    assert "head_dim" in _lib.last_error()
