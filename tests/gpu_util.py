"""GPU test helpers (torch only moves bytes; all compute goes through the C ABI)."""
import numpy as np
import torch

import oracle


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def f16_cache(rows_f32):
    """Device f16 cache holding the RNE image of rows_f32, and its f32 value."""
    bits = oracle.f32_to_f16_bits(rows_f32)
    t = torch.from_numpy(bits.view(np.int16)).view(torch.float16).cuda()
    return t, oracle.f16_bits_to_f32(bits)
