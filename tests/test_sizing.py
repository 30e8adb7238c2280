"""CPU: the decode cache sizing rules (sf37kv_sliding_cache_cap,
sf37kv_sliding_prefill_cap, sf37kv_kv_cache_bytes, sf37kv_plan_caches,
sf37kv_prefill_default_chunk) against the reference engine's own helpers
(sf37.c:3067-3096, 3189-3211, 5131-5140, built from its sources into
oracle/_ref/libsf37ref_sizing.so), and the managed-memory policy's device
branch (sf37_cuda.cu:1766-1800) on given free/total bytes."""
import ctypes

import pytest

import oracle
from sf37_b200 import _lib

GIB = 1 << 30
CTX = [1, 2, 100, 511, 512, 513, 700, 1024, 4096, 4607, 4608, 8192, 8704, 9000, 32768, 65536, 131072,
       262144]
CHUNK = [0, 1, 255, 256, 512, 1024, 2048, 4096, 7680, 7681, 8192, 262144]

needs_ref = pytest.mark.skipif(not oracle.ref_sizing_available(), reason="oracle/_ref sizing library not built")


@needs_ref
def test_sliding_caps_match_reference():
    L, R = _lib.lib(), oracle.ref_sizing()
    for ctx in CTX:
        for chunk in CHUNK:
            cap = L.sf37kv_sliding_cache_cap(ctx, chunk)
            assert cap == R.sf37ref_sliding_cache_cap(ctx, chunk), (ctx, chunk)
            assert L.sf37kv_sliding_prefill_cap(ctx, cap) == R.sf37ref_sliding_prefill_cap(ctx, cap), (ctx, cap)
        for cap in (0, 1, 512, 513, 4608, 8192):
            assert L.sf37kv_sliding_prefill_cap(ctx, cap) == R.sf37ref_sliding_prefill_cap(ctx, cap), (ctx, cap)


@needs_ref
def test_kv_bytes_and_plan_match_reference():
    L, R = _lib.lib(), oracle.ref_sizing()
    for cap in (1, 512, 4608, 32768, 262144):
        assert L.sf37kv_kv_cache_bytes(cap, 8, 128, 4) == R.sf37ref_decode_kv_bytes_for_cap(cap)
        assert L.sf37kv_kv_cache_bytes(cap, 8, 128, 2) * 2 == R.sf37ref_decode_kv_bytes_for_cap(cap)
    for ctx, chunk in ((32768, 4096), (65536, 2048), (262144, 4096), (300, 512), (1 << 20, 1024)):
        plan = _lib.CachePlan()
        assert L.sf37kv_plan_caches(ctx, chunk, 45, 8, 128, 4, ctypes.byref(plan)) == 0
        ctx_c = min(ctx, 262144)
        scap = R.sf37ref_sliding_cache_cap(ctx_c, chunk)
        assert plan.ctx_size == ctx_c and plan.sliding_cap == scap
        assert plan.prefill_cap == max(1, R.sf37ref_sliding_prefill_cap(ctx_c, scap))
        total = 0
        for il in range(45):
            full = R.sf37ref_layer_is_full(il)
            assert plan.sliding[il] == (0 if full else 1)
            assert plan.cap[il] == (ctx_c if full else scap)
            total += R.sf37ref_decode_kv_bytes_for_cap(plan.cap[il])
        assert plan.kv_cache_bytes == total
        assert (plan.full_layers, plan.sliding_layers) == (12, 33)


def test_prefill_default_chunk_tiers():
    # sf37.c:5131-5140 (the environment override is the caller's)
    L = _lib.lib()
    for free, want in ((0, 512), (6 * GIB - 1, 512), (6 * GIB, 1024), (12 * GIB, 2048), (24 * GIB - 1, 2048),
                       (24 * GIB, 4096), (180 * GIB, 4096)):
        assert L.sf37kv_prefill_default_chunk(free) == want


def test_managed_policy_device_branch():
    # The branch that needs the device's free/total memory, on given values.
    L = _lib.lib()
    total = 180 * GIB
    for kv in (0, 1, 4 * GIB, 8 * GIB - 1, 8 * GIB):
        for ctx in (0, 8 * GIB - 1, 8 * GIB, 20 * GIB, 100 * GIB, 200 * GIB):
            for free in (0, 10 * GIB, 60 * GIB, 150 * GIB, 180 * GIB):
                for tot in (16 * GIB, total, 400 * GIB):
                    want = oracle.managed_kv_policy(kv, ctx, free, tot)
                    assert L.sf37kv_managed_kv_policy(kv, ctx, free, tot) == want, (kv, ctx, free, tot)


def test_plan_rejects():
    L = _lib.lib()
    plan = _lib.CachePlan()
    assert L.sf37kv_plan_caches(1024, 512, 65, 8, 128, 2, ctypes.byref(plan)) == 1
    assert L.sf37kv_plan_caches(1024, 512, 4, 8, 128, 3, ctypes.byref(plan)) == 1
    assert L.sf37kv_plan_caches(1024, 512, 4, 8, 128, 2, None) == 1


def test_native_prefill_rejects_a_ring_too_small_for_the_chunk():
    # A 768-row sliding ring holds a chunk of up to 768 - 512 + 1 tokens
    # whose first token still sees its whole 512-row window; one more token
    # is rejected before any launch (fake device pointers are never touched).
    L = _lib.lib()
    c = _lib.Cache(256, 256, 768, 1, 512, 0)
    args = lambda n: (ctypes.byref(c), 256, 0, None, 256, 2000, n, 64, 8, 128, 2, None)
    assert L.sf37kv_prefill(*args(258)) == 1
    assert "sliding ring" in _lib.last_error()
