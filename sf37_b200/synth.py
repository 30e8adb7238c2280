"""Seeded synthetic inputs shared by the tests, the smoke run and the bench.

Host-side generator (small cases, bit-identical wherever numpy runs):
splitmix64 counter stream -> Box-Muller -> N(0, 1) float32, the f16 caches
being the IEEE round-to-nearest-even image of those values.  Large bench
inputs use torch's seeded CUDA generator instead (same distribution).
"""
import numpy as np

_GOLD = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + np.arange(1, n + 1, dtype=np.uint64) * _GOLD
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def normal(seed: int, shape) -> np.ndarray:
    """N(0,1) float32 of the given shape from stream `seed`."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    z = splitmix64(seed, m)
    u1 = ((z >> np.uint64(40)).astype(np.float64) + 0.5) / 16777216.0
    u2 = ((z & np.uint64(0xFFFFFF)).astype(np.float64) + 0.5) / 16777216.0
    r = np.sqrt(-2.0 * np.log(u1))
    t = 2.0 * np.pi * u2
    out = np.empty(2 * m, np.float64)
    out[0::2] = r * np.cos(t)
    out[1::2] = r * np.sin(t)
    return out[:n].astype(np.float32).reshape(shape)


def normal_f16(seed: int, shape) -> np.ndarray:
    """f16 (as numpy float16) RNE image of normal(seed, shape)."""
    return normal(seed, shape).astype(np.float16)


def cfg1_inputs(seed: int = 0, cached: int = 2048, q_heads: int = 64, kv_heads: int = 8,
                head_dim: int = 128):
    """`cached` f16 K/V rows, the new fp32 K/V row appended
    at position `cached`, an fp32 query; streams derived from `seed`."""
    kv_dim = kv_heads * head_dim
    k = normal_f16(seed * 16 + 1, (cached, kv_dim))
    v = normal_f16(seed * 16 + 2, (cached, kv_dim))
    k_new = normal(seed * 16 + 3, (kv_dim,))
    v_new = normal(seed * 16 + 4, (kv_dim,))
    q = normal(seed * 16 + 5, (q_heads, head_dim))
    gate = normal(seed * 16 + 6, (q_heads,))
    return k, v, k_new, v_new, q, gate


def q8_0_weights(seed, out_dim, in_dim):
    """Q8_0 weight rows [out_dim][in_dim/32 blocks x 34 bytes]: f16 scales in
    [1e-3, 2e-2) and int8 codes uniform in [-127, 127] (the range the
    reference's quantizer emits)."""
    rng = np.random.default_rng(seed)
    nb = in_dim // 32
    w = np.empty((out_dim, nb, 34), np.uint8)
    w[:, :, :2] = (rng.random((out_dim, nb)) * 0.019 + 0.001).astype(np.float16).view(np.uint8).reshape(
        out_dim, nb, 2)
    w[:, :, 2:] = rng.integers(-127, 128, (out_dim, nb, 32)).astype(np.int8).view(np.uint8)
    return w.reshape(out_dim, nb * 34)
