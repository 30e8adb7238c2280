"""GPU: the managed-KV-cache decision through the drop-in entry point
(sf37_cuda_should_use_managed_kv_cache, which reads the device's free and
total memory) equals the reference's own compiled function on the same
device and the policy restated on torch's view of the same memory."""
import pytest
import torch

import oracle
from sf37_b200 import _lib

pytestmark = pytest.mark.gpu
GIB = 1 << 30


def test_managed_policy_live_device_matches_reference():
    L = _lib.lib()
    R = oracle.ref_cuda() if oracle.ref_cuda_available() else None
    torch.cuda.init()
    free, total = torch.cuda.mem_get_info()
    cases = [(0, 0), (1 * GIB, 1 * GIB), (8 * GIB, 0), (4 * GIB, 8 * GIB), (4 * GIB, free - 60 * GIB),
             (4 * GIB, free - 20 * GIB), (4 * GIB, free - 1 * GIB), (4 * GIB, free + GIB), (7 * GIB, 500 * GIB)]
    for kv, ctx in cases:
        ctx = max(ctx, 0)
        got = L.sf37_cuda_should_use_managed_kv_cache(kv, ctx)
        # free memory moves by at most a few MB between the calls; the cases
        # sit GiBs away from every threshold
        assert got == oracle.managed_kv_policy(kv, ctx, free, total), (kv, ctx)
        if R is not None:
            R.sf37_cuda_should_use_managed_kv_cache.restype = __import__("ctypes").c_int
            R.sf37_cuda_should_use_managed_kv_cache.argtypes = [__import__("ctypes").c_uint64] * 2
            assert got == R.sf37_cuda_should_use_managed_kv_cache(kv, ctx), (kv, ctx)
