"""CPU: the C-ABI library loads and exports every symbol include/*.h
declares; argument validation that returns before any CUDA call."""
import ctypes
import os
import re

import pytest

from sf37_b200 import _lib

INC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")


def _declared():
    names = set()
    for f in os.listdir(INC):
        if not f.endswith(".h"):
            continue
        src = open(os.path.join(INC, f)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(sf37\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = _declared()
    assert len(names) >= 38
    for n in sorted(names):
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, f"{n} not bound in sf37_b200._lib"


def test_bindings_cover_only_declared_symbols():
    assert set(_lib.SIGNATURES) <= _declared()


def test_row_bytes():
    L = _lib.lib()
    assert L.sf37kv_row_bytes(1024, 0, 64) == 4096
    assert L.sf37kv_row_bytes(1024, 1, 64) == 1088  # sf37.c:6628-6631


def test_managed_policy_fast_paths():
    # sf37_cuda.cu:1775-1785: the two branches decided without the device.
    L = _lib.lib()
    assert L.sf37_cuda_should_use_managed_kv_cache(0, 1 << 40) == 0
    assert L.sf37_cuda_should_use_managed_kv_cache(8 << 30, 0) == 1
    assert L.sf37_cuda_should_use_managed_kv_cache(1 << 30, 1 << 30) == 0


def test_dropin_rejects_bad_arguments_without_launching():
    L = _lib.lib()
    t = _lib.Tensor(None, 0)
    tp = ctypes.byref(t)
    # NULL tensors and inconsistent heads -> 0 (sf37_cuda.cu:3015-3017, 6382).
    assert L.sf37_cuda_attention_decode_heads(None, None, None, None, None, 1, 1, 8, 2, 128, 0, 0) == 0
    assert L.sf37_cuda_attention_decode_heads_at(tp, tp, tp, tp, tp, 0, 4, 6, 4, 128, 0, 0) == 0
    assert L.sf37_cuda_store_kv_cache_batch(tp, tp, tp, tp, 0, 0, 4, 1024) == 0
    # byte sizes too small -> 0
    assert L.sf37_cuda_store_kv_cache_batch(tp, tp, tp, tp, 0, 1, 4, 1024) == 0
    assert L.sf37_cuda_attention_prefill_heads(tp, tp, tp, tp, tp, 0, 0, 8, 8, 2, 128, 0, 0) == 0
    assert L.sf37_cuda_gqa_single_token_heads(tp, tp, tp, 6, 4, 128) == 0


def test_native_rejects_bad_dtype_and_format():
    L = _lib.lib()
    lay = (_lib.DecodeLayer * 1)()
    lay[0].cache.cap = 16
    lay[0].cache.k_cache = 16
    lay[0].cache.v_cache = 16
    lay[0].q = 16
    lay[0].out = 16
    assert L.sf37kv_decode(lay, 1, 8, 2, 128, 3, None) == 1  # EINVAL: dtype
    assert "dtype" in _lib.last_error()
    assert L.sf37kv_decode(lay, 1, 6, 4, 128, 2, None) == 1  # EINVAL: heads
    pk = (_lib.PackLayer * 1)()
    assert L.sf37kv_pack(None, pk, 1, 1024, 2, 7, 64, 1, None) == 1  # EINVAL: fmt
    assert L.sf37kv_pack(None, pk, 1, 1024, 2, 1, 48, 1, None) == 4  # EUNSUPPORTED: group


def test_gather_rejects_bad_descriptors_without_launching():
    L = _lib.lib()
    lay = (_lib.DecodeLayer * 1)()
    lay[0].cache.cap = 16
    lay[0].cache.k_cache = lay[0].cache.v_cache = lay[0].q = 16
    g = _lib.PeerGather()
    g.world, g.rank = 9, 0
    assert L.sf37kv_decode_gather(lay, 1, 8, 1, 128, 2, ctypes.byref(g), 1, None) == 1
    assert "world" in _lib.last_error()
    g.world, g.rank = 2, 2
    assert L.sf37kv_decode_gather(lay, 1, 8, 1, 128, 2, ctypes.byref(g), 1, None) == 1
    g.rank = 1
    g.peer_buf[0] = g.peer_flags[0] = 256
    # peer 1's buffer is NULL
    assert L.sf37kv_decode_gather(lay, 1, 8, 1, 128, 2, ctypes.byref(g), 1, None) == 1
    assert "peer 1" in _lib.last_error()
    g.peer_buf[1] = g.peer_flags[1] = 512
    # no done counter
    assert L.sf37kv_decode_gather(lay, 1, 8, 1, 128, 2, ctypes.byref(g), 1, None) == 1
    g.done_counter = 1024
    # zero layers would never raise the epoch flag
    assert L.sf37kv_decode_gather(lay, 0, 8, 1, 128, 2, ctypes.byref(g), 1, None) == 1
    assert "no layers" in _lib.last_error()
    # head_dim 64 has no gather kernel
    assert L.sf37kv_decode_gather(lay, 1, 8, 1, 64, 2, ctypes.byref(g), 1, None) == 4
    assert L.sf37kv_gather_wait(None, 1, None) == 1


def test_prep_and_oproj_reject_bad_arguments_without_launching():
    L = _lib.lib()
    lay = (_lib.DecodeLayer * 1)()
    lay[0].cache.cap = 16
    lay[0].cache.k_cache = lay[0].cache.v_cache = lay[0].q = lay[0].out = 256
    prep = (_lib.QkPrep * 1)()
    assert L.sf37kv_decode_prep(lay, None, 1, 64, 8, 128, 2, None) == 1  # prep NULL
    prep[0].q_norm = prep[0].k_norm = 512
    prep[0].rotary_dim = 63
    assert L.sf37kv_decode_prep(lay, prep, 1, 64, 8, 128, 2, None) == 1
    assert "rotary_dim" in _lib.last_error()
    prep[0].rotary_dim = 64
    prep[0].q_norm = 0
    assert L.sf37kv_decode_prep(lay, prep, 1, 64, 8, 128, 2, None) == 1
    assert L.sf37kv_decode_prep(lay, prep, 1, 64, 8, 64, 2, None) == 4  # head_dim 64
    # o_proj
    op = (_lib.OprojLayer * 1)(_lib.OprojLayer(256, 256, 256))
    assert L.sf37kv_oproj_q8_0(op, 1, 100, 8, None) == 4  # in_dim % 256
    op[0].x = 260
    assert L.sf37kv_oproj_q8_0(op, 1, 256, 8, None) == 1  # alignment
    g = _lib.PeerGather()
    g.world, g.rank = 0, 0
    assert L.sf37kv_oproj_q8_0_shard(op, 1, 256, 8, 272, ctypes.byref(g), 1, None) == 1
    assert L.sf37kv_oproj_reduce(ctypes.byref(g), 1, 8, 1, None, None) == 1
