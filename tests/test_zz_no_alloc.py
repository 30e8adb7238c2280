"""GPU: the allocation-free decode entry point (sf37kv_decode_noalloc).

Callers that cannot call cudaMalloc while decoding (a memory pool that owns
the whole device, allocations frozen after start-up) use this entry point;
its split-K scratch is a fixed device array inside the library.  These tests
call it through the C ABI, two calls in a row (every call reuses the same
array), and check:
  - the outputs against the CPU oracle (the reference's attention restated)
    and against the regular entry point sf37kv_decode on the same inputs;
  - the appended K/V rows (k_new / v_new set) bit for bit against
    sf37kv_decode's and the oracle's append;
  - that a rejected call leaves the caches untouched.
The file is named to be collected last."""
import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import _lib, kv
from tests.helpers import ATOL, RTOL, F32_TOL, assert_close

pytestmark = pytest.mark.gpu


def _state(dtype, specs, qh, kvh, seed):
    """Per layer: caches (filled N(0,1)), and two calls' q / gate / new rows."""
    kd = kvh * 128
    tdt = torch.float16 if dtype == kv.F16 else torch.float32
    out = []
    for i, (cap, pos, sliding) in enumerate(specs):
        g = torch.Generator(device="cuda")
        g.manual_seed(seed + i)
        L = dict(k_cache=torch.randn(cap, kd, device="cuda", generator=g).to(tdt),
                 v_cache=torch.randn(cap, kd, device="cuda", generator=g).to(tdt),
                 cap=cap, pos=pos, sliding=sliding, window=512,
                 calls=[dict(q=torch.randn(qh, 128, device="cuda", generator=g),
                             gate=torch.randn(qh, device="cuda", generator=g),
                             k_new=torch.randn(kd, device="cuda", generator=g),
                             v_new=torch.randn(kd, device="cuda", generator=g)) for _ in range(2)])
        out.append(L)
    return out


def _clone(state):
    return [dict(L, k_cache=L["k_cache"].clone(), v_cache=L["v_cache"].clone()) for L in state]


def _call(entry, state, call, qh, kvh, dtype, append):
    """One decode call of every layer at position pos + call."""
    descs, outs = [], []
    for L in state:
        c = L["calls"][call]
        o = torch.full((qh, 128), float("nan"), device="cuda")
        outs.append(o)
        descs.append(dict(k_cache=L["k_cache"], v_cache=L["v_cache"], cap=L["cap"], sliding=L["sliding"],
                          window=512, pos=L["pos"] + call, q=c["q"], gate=c["gate"], out=o,
                          k_new=c["k_new"] if append else None, v_new=c["v_new"] if append else None))
    arr = kv.decode_layers_desc(descs)
    rc = getattr(_lib.lib(), entry)(arr, len(arr), qh, kvh, 128, dtype, None)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs]


def _host_cache(t):
    a = t.cpu()
    return a.view(torch.int16).numpy().view(np.uint16) if a.dtype == torch.float16 else a.numpy()


def _oracle_call(host, L, call, qh, kvh, append):
    """The oracle's step: ring append (f16 RNE for f16 caches), then attention."""
    kd = kvh * 128
    c = L["calls"][call]
    pos = L["pos"] + call
    if append:
        oracle.store_kv_rows(host["k"], host["v"], c["k_new"].cpu().numpy()[None], c["v_new"].cpu().numpy()[None],
                             pos, 1, L["cap"], kd)
    return oracle.attention_decode_at(c["q"].cpu().numpy(), host["k"], host["v"], c["gate"].cpu().numpy(), pos,
                                      L["cap"], qh, kvh, 128, L["sliding"], 512)


CASES = [
    (kv.F16, 64, 8, [(2049, 2047, 0)]),
    (kv.F16, 64, 8, [(32769, 32767, 0), (512, 70000, 1), (9000, 8998, 0), (4096, 5000, 1)]),
    (kv.F16, 48, 4, [(20000, 19998, 0), (600, 1000, 1)]),       # group 12
    (kv.F32, 64, 8, [(6000, 5998, 0), (512, 3000, 1)]),
    (kv.F32, 40, 8, [(3000, 2998, 0)]),                         # group 5
]


@pytest.mark.parametrize("append", [False, True])
@pytest.mark.parametrize("dtype,qh,kvh,specs", CASES)
def test_noalloc_matches_oracle_and_regular_entry_twice(dtype, qh, kvh, specs, append):
    a = _state(dtype, specs, qh, kvh, seed=77)
    b = _clone(a)
    hosts = [dict(k=_host_cache(L["k_cache"]), v=_host_cache(L["v_cache"])) for L in a]
    tol = dict(atol=ATOL, rtol=RTOL) if dtype == kv.F16 else dict(atol=F32_TOL, rtol=1e-4)
    for call in range(2):
        got = _call("sf37kv_decode_noalloc", a, call, qh, kvh, dtype, append)
        reg = _call("sf37kv_decode", b, call, qh, kvh, dtype, append)
        for i, L in enumerate(a):
            want = _oracle_call(hosts[i], L, call, qh, kvh, append)
            assert np.isfinite(got[i]).all(), f"call {call} layer {i}: output not written"
            assert_close(got[i], want, what=f"oracle, call {call} layer {i}", **tol)
            assert_close(got[i], reg[i], what=f"sf37kv_decode, call {call} layer {i}", **tol)
    for i, (La, Lb) in enumerate(zip(a, b)):
        for n in ("k_cache", "v_cache"):
            ga = _host_cache(La[n])
            assert np.array_equal(ga, _host_cache(Lb[n])), f"layer {i} {n} differs from sf37kv_decode's"
            assert np.array_equal(ga, hosts[i][n[0]]), f"layer {i} {n} differs from the oracle's append"


def test_noalloc_many_layers_exercises_capacity():
    # 48 layers x 8K rows: the split plan must be coarsened to fit the fixed
    # partial buffer; results still match the regular entry point.
    a = _state(kv.F16, [(8192, 8190, 0)] * 48, 64, 8, seed=5)
    b = _clone(a)
    for call in range(2):
        got = _call("sf37kv_decode_noalloc", a, call, 64, 8, kv.F16, True)
        want = _call("sf37kv_decode", b, call, 64, 8, kv.F16, True)
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


@pytest.mark.parametrize("qh,kvh,hd", [(8, 2, 64), (64, 2, 128)])
def test_noalloc_rejected_call_leaves_caches_untouched(qh, kvh, hd):
    # k_new set, then a shape the entry point rejects (head_dim 64, or group
    # 32): nothing may be written, the appended row included.
    kd = kvh * hd
    kc = torch.randn(64, kd, device="cuda").half()
    vc = torch.randn(64, kd, device="cuda").half()
    k0, v0 = kc.clone(), vc.clone()
    arr = kv.decode_layers_desc([dict(k_cache=kc, v_cache=vc, cap=64, pos=10, q=torch.randn(qh, hd, device="cuda"),
                                      gate=None, out=torch.empty(qh, hd, device="cuda"),
                                      k_new=torch.randn(kd, device="cuda"), v_new=torch.randn(kd, device="cuda"))])
    assert _lib.lib().sf37kv_decode_noalloc(arr, 1, qh, kvh, hd, kv.F16, None) == 4
    torch.cuda.synchronize()
    assert torch.equal(kc, k0) and torch.equal(vc, v0)
