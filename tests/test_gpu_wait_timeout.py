"""GPU: the bounded waits give up cleanly.  A peer descriptor whose flags
nothing ever raises (both 'ranks' are buffers on this one GPU, and no rank
runs) makes sf37kv_gather_wait and sf37kv_oproj_reduce time out after about
two seconds: the kernel sets the device error flag to 2 and returns, and the
context stays usable.  No fault, trap or hang is involved."""
import ctypes
import time

import pytest
import torch

from sf37_b200 import _lib

pytestmark = pytest.mark.gpu


def _desc(buf_floats=64):
    L = _lib.lib()
    bufs = [L.sf37kv_dev_alloc(buf_floats * 4 + 1024) for _ in range(2)]
    assert all(bufs)
    g = _lib.PeerGather()
    for p in range(2):
        g.peer_buf[p] = bufs[p]
        g.peer_flags[p] = bufs[p] + buf_floats * 4
    g.my_flags = bufs[0] + buf_floats * 4
    g.done_counter = bufs[0] + buf_floats * 4 + 512
    g.world, g.rank = 2, 0
    return g, bufs


def test_gather_wait_times_out_and_reports():
    L = _lib.lib()
    g, bufs = _desc()
    assert L.sf37kv_device_error(1) in (0, 2)
    t0 = time.time()
    assert L.sf37kv_gather_wait(ctypes.byref(g), 1, None) == 0
    assert L.sf37kv_device_error(1) == 2  # synchronizes: the wait gave up
    assert 0.5 < time.time() - t0 < 30
    # the context is still usable
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 28.0
    assert L.sf37kv_device_error(0) == 0
    for b in bufs:
        L.sf37kv_dev_free(b)


def test_oproj_reduce_times_out_and_reports():
    L = _lib.lib()
    g, bufs = _desc(2 * 2 * 1 * 64)
    out = torch.empty(64, device="cuda")
    assert L.sf37kv_oproj_reduce(ctypes.byref(g), 1, 64, 3, out.data_ptr(), None) == 0
    assert L.sf37kv_device_error(1) == 2
    assert L.sf37kv_device_error(0) == 0
    for b in bufs:
        L.sf37kv_dev_free(b)
