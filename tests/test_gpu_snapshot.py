"""GPU parity: snapshot KV pack/restore, bit-exact with the reference
formats (raw f32 rows, sf37.c:7298-7320; int8-grouped payload rows,
sf37.c:6980-7010 with payload_encode_kv_row_i8_grouped 6633-6659)."""
import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import kv, synth
from tests.gpu_util import dev, f16_cache, host

pytestmark = pytest.mark.gpu


def _layers(dtype, specs, kd=1024, scale=1.0):
    out = []
    for i, (cap, first, rows) in enumerate(specs):
        kf = synth.normal(900 + i, (cap, kd)) * np.float32(scale)
        vf = synth.normal(950 + i, (cap, kd)) * np.float32(scale)
        if dtype == kv.F16:
            kc, _ = f16_cache(kf)
            vc, _ = f16_cache(vf)
            hk, hv = oracle.f32_to_f16_bits(kf), oracle.f32_to_f16_bits(vf)
        else:
            kc, vc, hk, hv = dev(kf), dev(vf), kf, vf
        out.append(dict(k_cache=kc, v_cache=vc, cap=cap, first_pos=first, rows=rows, hk=hk, hv=hv))
    return out


SPECS = [(64, 0, 64), (512, 70000 - 512, 512), (100, 37, 80), (8, 3, 0), (300, 1000, 1)]


@pytest.mark.parametrize("dtype", [kv.F32, kv.F16])
@pytest.mark.parametrize("fmt", [kv.FMT_RAW, kv.FMT_I8G])
def test_pack_bit_exact(dtype, fmt):
    Ls = _layers(dtype, SPECS)
    arr, total = kv.pack_layers_desc(Ls, 1024, fmt)
    buf = torch.empty(total, dtype=torch.uint8, device="cuda")
    kv.pack(buf, arr, 1024, dtype, fmt)
    got = host(buf)
    want = np.concatenate([oracle.pack_layer(L["hk"], L["hv"], L["first_pos"], L["rows"], L["cap"], 1024,
                                             fmt) for L in Ls])
    assert np.array_equal(got, want)
    if fmt == kv.FMT_I8G and oracle.ref_available():
        # the same rows through the reference's own compiled encoder
        rows = np.concatenate([oracle.f16_bits_to_f32(np.stack([L["hk"][(L["first_pos"] + r) % L["cap"]],
                                                                L["hv"][(L["first_pos"] + r) % L["cap"]]]))
                               if dtype == kv.F16 else
                               np.stack([L["hk"][(L["first_pos"] + r) % L["cap"]],
                                         L["hv"][(L["first_pos"] + r) % L["cap"]]])
                               for L in Ls for r in range(L["rows"])])
        assert np.array_equal(got.reshape(-1, 1088), oracle.ref_payload_encode_rows(rows))


@pytest.mark.parametrize("dtype", [kv.F32, kv.F16])
@pytest.mark.parametrize("fmt", [kv.FMT_RAW, kv.FMT_I8G])
def test_unpack_inverse(dtype, fmt):
    Ls = _layers(dtype, SPECS)
    arr, total = kv.pack_layers_desc(Ls, 1024, fmt)
    if fmt == kv.FMT_RAW:
        # finite f32 values
        src = (synth.normal(6, (total // 4,))).view(np.uint8).copy()
    else:
        rb = 1088
        rows = synth.normal(7, (total // rb, 1024))
        src = oracle.payload_encode_rows(rows).reshape(-1)
    kv.unpack(dev(src), arr, 1024, dtype, fmt)
    torch.cuda.synchronize()
    for i, L in enumerate(Ls):
        hk, hv = L["hk"].copy(), L["hv"].copy()
        off = arr[i].offset
        sec = src[off: off + 2 * L["rows"] * kv.row_bytes(1024, fmt)]
        oracle.unpack_layer(sec, hk, hv, L["first_pos"], L["rows"], L["cap"], 1024, fmt)
        gk = L["k_cache"].cpu()
        gv = L["v_cache"].cpu()
        if dtype == kv.F16:
            gk = gk.view(torch.int16).numpy().view(np.uint16)
            gv = gv.view(torch.int16).numpy().view(np.uint16)
        else:
            gk, gv = gk.numpy(), gv.numpy()
        assert np.array_equal(gk, hk) and np.array_equal(gv, hv)


@pytest.mark.parametrize("fmt", [kv.FMT_RAW, kv.FMT_I8G])
def test_pack_to_host_roundtrip(fmt):
    Ls = _layers(kv.F16, [(5000, 123, 5000), (512, 9000, 512)])
    arr, total = kv.pack_layers_desc(Ls, 1024, fmt)
    hbuf = np.empty(total, np.uint8)
    kv.pack_to_host(hbuf.ctypes.data, arr, 1024, kv.F16, fmt)
    want = np.concatenate([oracle.pack_layer(L["hk"], L["hv"], L["first_pos"], L["rows"], L["cap"], 1024,
                                             fmt) for L in Ls])
    assert np.array_equal(hbuf, want)
    if fmt == kv.FMT_RAW:
        # restore into zeroed caches reproduces the f16 caches exactly
        for L in Ls:
            L["k_cache"].zero_()
            L["v_cache"].zero_()
        kv.unpack_from_host(hbuf.ctypes.data, arr, 1024, kv.F16, fmt)
        for L in Ls:
            assert np.array_equal(L["k_cache"].cpu().view(torch.int16).numpy().view(np.uint16), L["hk"])


@pytest.mark.parametrize("fmt", [kv.FMT_RAW, kv.FMT_I8G])
def test_dropin_pack_rows(fmt):
    cap, first, rows = 520, 600, 500
    kf = synth.normal(41, (cap, 1024))
    vf = synth.normal(42, (cap, 1024))
    dk, dv = dev(kf), dev(vf)
    rb = kv.row_bytes(1024, fmt)
    hbuf = np.empty(2 * rows * rb, np.uint8)
    assert kv.kv_pack_rows(hbuf, dk, dv, first, rows, cap, 1024, fmt)
    assert np.array_equal(hbuf, oracle.pack_layer(kf, vf, first, rows, cap, 1024, fmt))
    dk.zero_()
    dv.zero_()
    assert kv.kv_unpack_rows(hbuf, dk, dv, first, rows, cap, 1024, fmt)
    hk = np.zeros_like(kf)
    hv = np.zeros_like(vf)
    oracle.unpack_layer(hbuf, hk, hv, first, rows, cap, 1024, fmt)
    assert np.array_equal(host(dk), hk) and np.array_equal(host(dv), hv)


@pytest.mark.parametrize("dtype", [kv.F32, kv.F16])
def test_pack_i8_special_values(dtype):
    # all-zero groups, +-inf / NaN (skipped by the max, encoded as 0), huge
    # and tiny magnitudes, exact .5 ties: bit-exact with the oracle
    cap, kd = 40, 1024
    rng = np.random.default_rng(3)
    k = (rng.standard_normal((cap, kd)) * 3).astype(np.float32)
    v = (rng.standard_normal((cap, kd)) * 0.01).astype(np.float32)
    k[0, :64] = 0
    k[1, 5] = np.inf
    k[1, 70] = -np.inf
    k[2, 3] = np.nan
    k[2, 64:128] = np.nan
    k[3, :] = 60000.0 * np.sign(rng.standard_normal(kd))
    k[4, :] = 1e-6
    v[5, :64] = np.arange(64) * 0.5 - 16  # many exact halves
    v[6, :] = -0.0
    if dtype == kv.F16:
        hk, hv = oracle.f32_to_f16_bits(k), oracle.f32_to_f16_bits(v)
        kc = torch.from_numpy(hk.view(np.float16)).cuda()
        vc = torch.from_numpy(hv.view(np.float16)).cuda()
    else:
        hk, hv = k, v
        kc, vc = dev(k), dev(v)
    L = [dict(k_cache=kc, v_cache=vc, cap=cap, first_pos=0, rows=cap)]
    arr, total = kv.pack_layers_desc(L, kd, kv.FMT_I8G)
    buf = torch.empty(total, dtype=torch.uint8, device="cuda")
    kv.pack(buf, arr, kd, dtype, kv.FMT_I8G)
    want = oracle.pack_layer(hk, hv, 0, cap, cap, kd, kv.FMT_I8G)
    assert np.array_equal(host(buf), want)


@pytest.mark.parametrize("dtype", [kv.F16, kv.F32])
@pytest.mark.parametrize("fmt", [kv.FMT_RAW, kv.FMT_I8G])
def test_kv_head_slices_fill_one_record(dtype, fmt):
    # N GPUs' KV-head slices written into one full-layout record equal the
    # record packed from the full caches; restoring each slice from the
    # record equals restoring the full caches and taking its columns.
    from sf37_b200 import _lib
    Ls = _layers(dtype, [(300, 1000, 300), (64, 0, 40), (90, 17, 90)])
    arr, total = kv.pack_layers_desc(Ls, 1024, fmt)
    whole = np.empty(total, np.uint8)
    kv.pack_to_host(whole.ctypes.data, arr, 1024, dtype, fmt)
    for n in (2, 4, 8):
        kd = 1024 // n
        rec = np.full(total, 0xAB, np.uint8)
        for r in range(n):
            sl = [dict(k_cache=L["k_cache"][:, r * kd:(r + 1) * kd].contiguous(),
                       v_cache=L["v_cache"][:, r * kd:(r + 1) * kd].contiguous()) for L in Ls]
            sarr = (_lib.PackLayer * len(Ls))()
            for i, L in enumerate(Ls):
                sarr[i] = _lib.PackLayer(kv.cache_desc(sl[i]["k_cache"], sl[i]["v_cache"], L["cap"]), L["first_pos"],
                                         L["rows"], arr[i].offset)
            assert _lib.lib().sf37kv_pack_slice_to_host(rec.ctypes.data, sarr, len(Ls), kd, 1024, r * kd, dtype,
                                                        fmt, 64, 1) == 0, _lib.last_error()
            if r == n - 1:
                assert np.array_equal(rec, whole), n
            # restore this slice from the full record into zeroed slice caches
            for s in sl:
                s["k_cache"].zero_()
                s["v_cache"].zero_()
            assert _lib.lib().sf37kv_unpack_slice_from_host(whole.ctypes.data, sarr, len(Ls), kd, 1024, r * kd,
                                                            dtype, fmt, 64) == 0, _lib.last_error()
            torch.cuda.synchronize()
            for i, L in enumerate(Ls):
                full_k = torch.zeros_like(L["k_cache"])
                full_v = torch.zeros_like(L["v_cache"])
                one = [dict(k_cache=full_k, v_cache=full_v, cap=L["cap"], first_pos=L["first_pos"], rows=L["rows"])]
                oarr, _ = kv.pack_layers_desc(one, 1024, fmt)
                sec = 2 * L["rows"] * kv.row_bytes(1024, fmt)
                part = np.ascontiguousarray(whole[arr[i].offset:arr[i].offset + sec])
                kv.unpack_from_host(part.ctypes.data, oarr, 1024, dtype, fmt)
                torch.cuda.synchronize()
                assert torch.equal(sl[i]["k_cache"], full_k[:, r * kd:(r + 1) * kd])
                assert torch.equal(sl[i]["v_cache"], full_v[:, r * kd:(r + 1) * kd])


def test_kv_head_slice_spans_several_chunks():
    # A slice record larger than three 64 MiB staging chunks (and far more
    # than 4096 rows, so several host threads scatter): one KV head of a
    # 200000-row f16 layer, raw f32 format.  Exercises the double-buffered
    # pipeline (scatter of chunk c-1 while chunk c packs; the in-use wait on
    # restore) against pack_to_host / unpack_from_host of the full caches.
    from sf37_b200 import _lib
    rows, kd, full = 200000, 128, 1024
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    k = torch.randn(rows, full, device="cuda", generator=g).half()
    v = torch.randn(rows, full, device="cuda", generator=g).half()
    L = [dict(k_cache=k, v_cache=v, cap=rows, first_pos=0, rows=rows)]
    arr, total = kv.pack_layers_desc(L, full, kv.FMT_RAW)
    assert 2 * rows * 4 * kd > 3 * (64 << 20)
    whole = np.empty(total, np.uint8)
    kv.pack_to_host(whole.ctypes.data, arr, full, kv.F16, kv.FMT_RAW)
    r = 5
    ks = k[:, r * kd:(r + 1) * kd].contiguous()
    vs = v[:, r * kd:(r + 1) * kd].contiguous()
    sarr = (_lib.PackLayer * 1)(_lib.PackLayer(kv.cache_desc(ks, vs, rows), 0, rows, 0))
    rec = np.zeros(total, np.uint8)
    assert _lib.lib().sf37kv_pack_slice_to_host(rec.ctypes.data, sarr, 1, kd, full, r * kd, kv.F16, kv.FMT_RAW,
                                                64, 1) == 0, _lib.last_error()
    # only this head's columns of every row were written
    rb = full * 4
    recv = rec.reshape(2 * rows, rb)
    wv = whole.reshape(2 * rows, rb)
    assert np.array_equal(recv[:, 4 * r * kd:4 * (r + 1) * kd], wv[:, 4 * r * kd:4 * (r + 1) * kd])
    assert not recv[:, :4 * r * kd].any() and not recv[:, 4 * (r + 1) * kd:].any()
    ks.zero_()
    vs.zero_()
    assert _lib.lib().sf37kv_unpack_slice_from_host(whole.ctypes.data, sarr, 1, kd, full, r * kd, kv.F16,
                                                    kv.FMT_RAW, 64) == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.equal(ks, k[:, r * kd:(r + 1) * kd]) and torch.equal(vs, v[:, r * kd:(r + 1) * kd])
