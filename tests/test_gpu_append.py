"""GPU parity: K/V append (ring slot (pos0+t) % cap), bit-exact with the
oracle (sf37_cuda.cu:6355-6401; f16: IEEE round-to-nearest-even)."""
import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import kv, synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("pos0,n_tok,cap,kv_dim", [(0, 1, 4, 1024), (2, 3, 8, 256), (5, 9, 4, 1024),
                                                    (2048, 1, 4096, 1024), (100, 37, 64, 1024),
                                                    (7, 5, 6, 6)])
def test_dropin_store_f32_bit_exact(pos0, n_tok, cap, kv_dim):
    k = synth.normal(1 + pos0, (n_tok, kv_dim))
    v = synth.normal(2 + pos0, (n_tok, kv_dim))
    kc0 = synth.normal(3, (cap, kv_dim))
    vc0 = synth.normal(4, (cap, kv_dim))
    dkc, dvc = dev(kc0), dev(vc0)
    assert kv.store_kv_cache_batch(dkc, dvc, dev(k), dev(v), pos0, n_tok, cap, kv_dim)
    kc, vc = kc0.copy(), vc0.copy()
    oracle.store_kv_rows(kc, vc, k, v, pos0, n_tok, cap, kv_dim)
    assert np.array_equal(host(dkc), kc)
    assert np.array_equal(host(dvc), vc)


def test_native_append_f16_multilayer_bit_exact():
    kv_dim, cap = 1024, 40
    layers, ref = [], []
    for l in range(5):
        n_tok = [1, 3, 17, 40, 2][l]
        pos0 = [0, 39, 77, 5, 1000][l]
        k = synth.normal(10 + l, (n_tok, kv_dim)) * np.float32(50.0)
        v = synth.normal(20 + l, (n_tok, kv_dim)) * np.float32(1e-4)
        kc = torch.zeros(cap, kv_dim, dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        layers.append(dict(k_cache=kc, v_cache=vc, cap=cap, pos0=pos0, n_tok=n_tok, k=dev(k), v=dev(v)))
        hk = np.zeros((cap, kv_dim), np.uint16)
        hv = np.zeros((cap, kv_dim), np.uint16)
        oracle.store_kv_rows(hk, hv, k, v, pos0, n_tok, cap, kv_dim)
        ref.append((hk, hv))
    kv.append(layers, kv_dim, kv.F16)
    torch.cuda.synchronize()
    for L, (hk, hv) in zip(layers, ref):
        assert np.array_equal(L["k_cache"].cpu().view(torch.int16).numpy().view(np.uint16), hk)
        assert np.array_equal(L["v_cache"].cpu().view(torch.int16).numpy().view(np.uint16), hv)


def test_append_f16_special_values():
    kv_dim = 16
    k = np.array([[65504, 65519, 65520, 1e9, -1e9, 6e-8, 2.98e-8, -0.0, 0.0, 1e-5, 0.1, 1.0 / 3,
                   np.inf, -np.inf, 5.96e-8, 1.5e-7]], np.float32)
    kc = torch.zeros(2, kv_dim, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    kv.append([dict(k_cache=kc, v_cache=vc, cap=2, pos0=1, n_tok=1, k=dev(k), v=dev(k))], kv_dim, kv.F16)
    got = kc.cpu().view(torch.int16).numpy().view(np.uint16)[1]
    assert np.array_equal(got, oracle.f32_to_f16_bits(k[0]))
