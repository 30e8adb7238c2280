"""Shared test helpers: tolerances and comparisons."""
import numpy as np

# attention outputs within max-abs 2e-3 and rel 1e-2
# (fp32 accumulate) of the reference; an element passes if either holds.
ATOL = 2e-3
RTOL = 1e-2
# The reference's own CUDA tests use 2e-5 .. 6e-5 on small integer-pattern
# fp32 inputs (tests/test_sf37_cuda_ops.cu:302-347, 1147); the fp32 cache
# path is held to that.
F32_TOL = 6e-5


def assert_close(got, want, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, (got.shape, want.shape)
    diff = np.abs(got - want)
    bad = (diff > atol) & (diff > rtol * np.abs(want))
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, diff, 0)), diff.shape)
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} elements out of tolerance; "
                             f"worst at {i}: got {got[i]} want {want[i]} (max diff {diff.max():.3g})")
    return float(diff.max())
