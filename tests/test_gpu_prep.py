"""GPU: decode with the q/k head norm + RoPE fused in (sf37kv_decode_prep)
against the oracle (the reference's CPU head_rms_norm_weight1 +
apply_rope_one, then the append and attention): the appended K row within
ulp-scale bounds, the attention output within the attention tolerance."""
import numpy as np
import pytest
import torch

import oracle
from sf37_b200 import kv, synth
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu
QH, KVH, HD = 64, 8, 128
# (rotary_dim, theta, llama3) of full (il % 4 == 0) and sliding layers, sf37.c:1983-1993
FULL, SLIDING = (64, 5e6, 1), (128, 1e4, 0)


def _bf16(seed):
    w = (synth.normal(seed, (HD,)) * 0.3).astype(np.float32)
    return (w.view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("f16,pos,qh", [(True, 0, 64), (True, 700, 64), (True, 4999, 64), (False, 0, 64),
                                         (False, 700, 64), (False, 4999, 64), (True, 3000, 96), (False, 600, 96)])
def test_decode_prep_matches_oracle(f16, pos, qh):
    # qh 96: the real model's sliding layers (group 12)
    QH = qh
    layers = 4
    caps = [5000, 512, 512, 512]
    params = [FULL, SLIDING, SLIDING, SLIDING]
    descs, preps, keep, want = [], [], [], []
    for l in range(layers):
        cap = caps[l]
        k = synth.normal(100 + l, (cap, KVH * HD))
        v = synth.normal(200 + l, (cap, KVH * HD))
        if f16:
            k = oracle.f32_to_f16_bits(k)
            v = oracle.f32_to_f16_bits(v)
        q = synth.normal(300 + l, (QH, HD)) * 2
        kn = synth.normal(400 + l, (KVH * HD,)) * 2
        vn = synth.normal(500 + l, (KVH * HD,))
        gate = synth.normal(600 + l, (QH,))
        qw, kw = _bf16(700 + l), _bf16(800 + l)
        rot, th, ll = params[l]
        # oracle: prepare, append, attend
        qp = oracle.qk_prep(q, qw, rot, th, ll, pos)
        kp = oracle.qk_prep(kn.reshape(KVH, HD), kw, rot, th, ll, pos).reshape(-1)
        ke, ve = k.copy(), v.copy()
        oracle.store_kv_rows(ke, ve, kp[None], vn[None], pos, 1, cap, KVH * HD)
        out_w = oracle.attention_decode_at(qp, ke, ve, gate, pos, cap, QH, KVH, HD, sliding=int(l % 4 != 0))
        want.append((kp, out_w))
        t = dict(k_cache=torch.from_numpy(k.view(np.float16) if f16 else k).cuda(),
                 v_cache=torch.from_numpy(v.view(np.float16) if f16 else v).cuda(),
                 q=torch.from_numpy(q).cuda(), gate=torch.from_numpy(gate).cuda(),
                 k_new=torch.from_numpy(kn).cuda(), v_new=torch.from_numpy(vn).cuda(),
                 out=torch.empty(QH, HD, device="cuda"),
                 qw=torch.from_numpy(qw.view(np.int16)).cuda(), kw=torch.from_numpy(kw.view(np.int16)).cuda())
        keep.append(t)
        descs.append(dict(k_cache=t["k_cache"], v_cache=t["v_cache"], cap=cap, sliding=l % 4 != 0, window=512,
                          pos=pos, q=t["q"], gate=t["gate"], out=t["out"], k_new=t["k_new"], v_new=t["v_new"]))
        preps.append(dict(q_norm=t["qw"], k_norm=t["kw"], rotary_dim=rot, theta=th, llama3=ll, eps=1e-5))
    q_before = [t["q"].clone() for t in keep]
    kv.decode_prep(descs, preps, QH, KVH, HD, kv.F16 if f16 else kv.F32)
    torch.cuda.synchronize()
    for l in range(layers):
        t, (kp, out_w) = keep[l], want[l]
        row = t["k_cache"][pos % caps[l]].float().cpu().numpy()
        if f16:
            # one f16 rounding of a value within ulp-scale bounds of the oracle
            np.testing.assert_allclose(row, oracle.f16_bits_to_f32(oracle.f32_to_f16_bits(kp)), rtol=1e-3,
                                       atol=1e-6)
        else:
            np.testing.assert_allclose(row, kp, rtol=1e-6, atol=2e-6)
        assert_close(t["out"].cpu().numpy(), out_w, what=f"layer {l}")
        assert torch.equal(t["q"], q_before[l])  # inputs are not modified


def test_decode_prep_rejects_bad_arguments():
    from sf37_b200 import _lib
    k = torch.zeros(16, KVH * HD, dtype=torch.float16, device="cuda")
    q = torch.zeros(QH, HD, device="cuda")
    w = torch.zeros(HD, dtype=torch.int16, device="cuda")
    d = [dict(k_cache=k, v_cache=k, cap=16, pos=3, q=q, out=q)]
    with pytest.raises(RuntimeError, match="rotary_dim"):
        kv.decode_prep(d, [dict(q_norm=w, k_norm=w, rotary_dim=129, theta=1e4)], QH, KVH, HD, kv.F16)
    with pytest.raises(RuntimeError, match="rotary_dim"):
        kv.decode_prep(d, [dict(q_norm=w, k_norm=w, rotary_dim=63, theta=1e4)], QH, KVH, HD, kv.F16)
    assert _lib.lib().sf37kv_decode_prep(kv.decode_layers_desc(d), None, 1, QH, KVH, HD, kv.F16, None) == 1
