"""GPU: BASELINE sizes, checked through properties that do not need the
oracle to process everything (plus sampled oracle checks).

* config 2 (48 x 32769 rows, f16): decode of all layers in one call equals
  the per-layer calls; two layers are checked against the oracle in full.
* config 5b (32768-token snapshot, 8 of 48 layers to bound host memory):
  raw pack -> restore into zeroed caches reproduces the caches bit for bit;
  int8 pack bytes and restored rows equal the reference encoder / the
  oracle decoder on sampled rows.
* config 4 (8192-token chunk on 24576, one layer): sampled tokens against
  the oracle (the full oracle would be ~10^13 flops).
"""
import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import kv
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


def _f16_bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_cfg2_batched_equals_per_layer_and_oracle():
    L, cap = 48, 32769
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    ks = [torch.randn(cap, 1024, device="cuda", generator=g).half() for _ in range(L)]
    vs = [torch.randn(cap, 1024, device="cuda", generator=g).half() for _ in range(L)]
    q = torch.randn(L, 64, 128, device="cuda", generator=g)
    gate = torch.randn(L, 64, device="cuda", generator=g)
    out_b = torch.empty(L, 64, 128, device="cuda")
    out_l = torch.empty(L, 64, 128, device="cuda")
    kv.decode([dict(k_cache=ks[l], v_cache=vs[l], cap=cap, pos=cap - 1, q=q[l], gate=gate[l], out=out_b[l])
               for l in range(L)], 64, 8, 128, kv.F16)
    for l in range(L):
        kv.decode([dict(k_cache=ks[l], v_cache=vs[l], cap=cap, pos=cap - 1, q=q[l], gate=gate[l], out=out_l[l])],
                  64, 8, 128, kv.F16)
    torch.cuda.synchronize()
    assert_close(out_b.cpu().numpy(), out_l.cpu().numpy(), atol=1e-5, rtol=1e-4, what="batched vs per-layer")
    for l in (0, 47):
        want = oracle.attention_decode_at(q[l].cpu().numpy(), oracle.f16_bits_to_f32(_f16_bits(ks[l])),
                                          oracle.f16_bits_to_f32(_f16_bits(vs[l])), gate[l].cpu().numpy(),
                                          cap - 1, cap, 64, 8, 128)
        assert_close(out_b[l].cpu().numpy(), want, what=f"layer {l}")


def test_cfg5b_snapshot_roundtrip():
    L, rows = 8, 32768
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    layers = [dict(k_cache=torch.randn(rows, 1024, device="cuda", generator=g).half(),
                   v_cache=torch.randn(rows, 1024, device="cuda", generator=g).half(),
                   cap=rows, first_pos=0, rows=rows) for _ in range(L)]
    keep = [(_f16_bits(x["k_cache"]), _f16_bits(x["v_cache"])) for x in layers]
    # raw: pack to host, zero the caches, restore, compare bits
    arr, total = kv.pack_layers_desc(layers, 1024, kv.FMT_RAW)
    host = np.empty(total, np.uint8)
    kv.pack_to_host(host.ctypes.data, arr, 1024, kv.F16, kv.FMT_RAW)
    for x in layers:
        x["k_cache"].zero_()
        x["v_cache"].zero_()
    kv.unpack_from_host(host.ctypes.data, arr, 1024, kv.F16, kv.FMT_RAW)
    for x, (hk, hv) in zip(layers, keep):
        assert np.array_equal(_f16_bits(x["k_cache"]), hk) and np.array_equal(_f16_bits(x["v_cache"]), hv)
    # sampled rows equal the oracle's section bytes
    rb = 4096
    for li in (0, L - 1):
        sec = host[arr[li].offset: arr[li].offset + 2 * rows * rb].reshape(rows, 2, rb)
        for r in (0, 1, 12345, rows - 1):
            want = oracle.pack_layer(keep[li][0][r:r + 1], keep[li][1][r:r + 1], 0, 1, 1, 1024, 0)
            assert np.array_equal(sec[r].reshape(-1), want)
    # int8: pack -> decode into caches -> pack again is the same bytes
    arr8, total8 = kv.pack_layers_desc(layers, 1024, kv.FMT_I8G)
    h8 = np.empty(total8, np.uint8)
    kv.pack_to_host(h8.ctypes.data, arr8, 1024, kv.F16, kv.FMT_I8G)
    if oracle.ref_available():
        k0 = oracle.f16_bits_to_f32(keep[0][0][:64])
        got = h8[:2 * 64 * 1088].reshape(64, 2, 1088)[:, 0]
        assert np.array_equal(got, oracle.ref_payload_encode_rows(k0))
    f32layers = [dict(k_cache=torch.empty(rows, 1024, device="cuda"), v_cache=torch.empty(rows, 1024, device="cuda"),
                      cap=rows, first_pos=0, rows=rows) for _ in range(2)]
    arr_f32, _ = kv.pack_layers_desc(f32layers, 1024, kv.FMT_I8G)
    kv.unpack_from_host(h8.ctypes.data, arr_f32, 1024, kv.F32, kv.FMT_I8G)
    # restored rows are exactly the oracle's decode of the payload rows
    sec = h8[:2 * 2 * rows * 1088].reshape(2, rows, 2, 1088)
    for li in (0, 1):
        for r in (0, 777, rows - 1):
            for kvi, name in ((0, "k_cache"), (1, "v_cache")):
                want = oracle.payload_decode_rows(sec[li, r, kvi], 1024)[0]
                got = f32layers[li][name][r].cpu().numpy()
                assert np.array_equal(got, want)


def test_cfg4_prefill_sampled_tokens():
    prefix, chunk, cap = 24576, 8192, 32768
    g = torch.Generator(device="cuda")
    g.manual_seed(13)
    kc = torch.randn(cap, 1024, device="cuda", generator=g).half()
    vc = torch.randn(cap, 1024, device="cuda", generator=g).half()
    q = torch.randn(chunk, 64, 128, device="cuda", generator=g).to(torch.bfloat16)
    gate = torch.randn(chunk, 64, device="cuda", generator=g)
    out = torch.empty(chunk, 64, 128, device="cuda")
    kv.prefill(kc, vc, cap, q, gate, out, prefix, chunk, 64, 8, 128, kv.F16)
    torch.cuda.synchronize()
    from sf37_b200 import _lib
    assert _lib.lib().sf37kv_device_error(1) == 0
    kf = oracle.f16_bits_to_f32(_f16_bits(kc))
    vf = oracle.f16_bits_to_f32(_f16_bits(vc))
    qf = q.float().cpu().numpy()
    gf = gate.cpu().numpy()
    got = out.cpu().numpy()
    for t in (0, 1, 4095, 8190, 8191):
        want = oracle.attention_prefill(qf, kf, vf, gf, prefix, chunk, cap, 64, 8, 128, t0=t, t1=t + 1)
        assert_close(got[t], want[t], what=f"token {t}")
