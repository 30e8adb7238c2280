"""CPU oracle for the KV-cache hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this package, and only as the checker or the timed CPU
baseline.  The shipped library never routes through it.

Two libraries live here:

* ``liboracle.so`` (built from ``oracle.c``): a C restatement of the
  reference's arithmetic, each function citing the reference file:line.
* ``_ref/libsf37ref.so`` (built from ``ref_harness.c`` + the reference's own
  ``sf37.c``/``sf37_ops.c``/... with the reference Makefile flags): the
  reference itself, used to pin the restatement and as the CPU baseline.
  ``_ref/libsf37ref_cuda.so`` is the reference's CUDA kernels built for
  sm_100a (fp32 caches), used as a GPU-side oracle and baseline.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# The reference source tree: $SF37_REF_DIR, else a "reference" directory next
# to this repository's root.
REF_DIR_DEFAULT = os.path.normpath(os.path.join(HERE, "..", "..", "reference"))

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_vp = ctypes.c_void_p
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_int = ctypes.c_int


def build(ref: bool = True, ref_cuda: bool = False) -> None:
    """Compile liboracle.so; with ``ref`` also the reference CPU library when
    the reference source tree is present (it is absent on GPU boxes, which use
    the prebuilt file)."""
    subprocess.check_call(["make", "-s", "-C", HERE, "oracle"])
    ref_dir = os.environ.get("SF37_REF_DIR", REF_DIR_DEFAULT)
    if os.path.isfile(os.path.join(ref_dir, "sf37.c")):
        targets = (["ref"] if ref else []) + (["ref-cuda"] if ref_cuda else [])
        for t in targets:
            subprocess.check_call(["make", "-s", "-C", HERE, t, f"REF_DIR={ref_dir}"])


def _ptr(a):
    return a.ctypes.data_as(_vp)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build(ref=False)
        L = ctypes.CDLL(path)
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16_array.argtypes = [_vp, _vp, _u64]
        L.orc_f16_to_f32_array.argtypes = [_vp, _vp, _u64]
        L.orc_store_kv_rows.argtypes = [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _int]
        args_attn = [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _int, _u32]
        L.orc_attention_decode_at.argtypes = args_attn
        L.orc_attention_decode_n.argtypes = args_attn
        L.orc_attention_prefill.argtypes = [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32,
                                            _u32, _u32, _int, _u32, _u32, _u32]
        L.orc_payload_row_bytes.restype = _u64
        L.orc_payload_row_bytes.argtypes = [_u32, _u32]
        L.orc_payload_encode_row.argtypes = [_vp, _u32, _u32, _int, _vp]
        L.orc_payload_decode_row.argtypes = [_vp, _u32, _u32, _vp]
        L.orc_pack_layer.argtypes = [_vp, _vp, _vp, _int, _u32, _u32, _u32, _u32, _int, _u32, _int]
        L.orc_unpack_layer.argtypes = [_vp, _vp, _vp, _int, _u32, _u32, _u32, _u32, _int, _u32]
        L.orc_q8_0_quantize.argtypes = [_vp, _vp, _vp, _u64]
        L.orc_q8_0_matvec.argtypes = [_vp, _vp, _u64, _u64, _vp]
        L.orc_qk_prep.argtypes = [_vp, _u32, _u32, _vp, _u32, ctypes.c_double, _int, _u32, ctypes.c_float]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libsf37ref.so"))


def ref():
    """The reference's own CPU code (compiled from its sources)."""
    global _ref
    if _ref is None:
        R = ctypes.CDLL(os.path.join(HERE, "_ref", "libsf37ref.so"))
        R.sf37ref_kv_cache_push_rows.argtypes = [_vp, _vp, _u32, ctypes.POINTER(_u32), _vp, _vp, _u32]
        R.sf37ref_attention_decode.argtypes = [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _int, _vp]
        R.sf37ref_payload_row_bytes.restype = _u64
        R.sf37ref_payload_row_bytes.argtypes = [_u32, _u32]
        R.sf37ref_payload_encode_rows.argtypes = [_vp, _u32, _u32, _u64, _vp]
        R.sf37ref_payload_decode_rows.argtypes = [_vp, _u32, _u32, _u64, _vp]
        R.sf37ref_decode_step_layers.restype = _int
        R.sf37ref_decode_step_layers.argtypes = [_vp] * 3 + [_u32] + [_vp] * 6 + [_u32, _u32, _u32]
        _ref = R
    return _ref


# ---------------------------------------------------------------- numpy API
def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_array(_ptr(x), _ptr(out), x.size)
    return out


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().orc_f16_to_f32_array(_ptr(h), _ptr(out), h.size)
    return out


def store_kv_rows(k_cache, v_cache, k, v, pos0, n_tok, cap, kv_dim):
    """In-place ring append; cache dtype float32 or uint16 (f16 bits)."""
    eb = 4 if k_cache.dtype == np.float32 else 2
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    lib().orc_store_kv_rows(_ptr(k_cache), _ptr(v_cache), _ptr(k), _ptr(v), pos0, n_tok, cap,
                            kv_dim, eb)


def _as_f32_cache(c):
    return f16_bits_to_f32(c) if c.dtype == np.uint16 else np.ascontiguousarray(c, np.float32)


def attention_decode_at(q, k_cache, v_cache, gate, pos, cap, q_heads, kv_heads, head_dim,
                        sliding=0, window=512):
    kc, vc = _as_f32_cache(k_cache), _as_f32_cache(v_cache)
    q = np.ascontiguousarray(q, np.float32)
    out = np.zeros((q_heads, head_dim), np.float32)
    g = None if gate is None else np.ascontiguousarray(gate, np.float32)
    lib().orc_attention_decode_at(_ptr(out), _ptr(q), _ptr(kc), _ptr(vc),
                                  None if g is None else _ptr(g), pos, cap, q_heads,
                                  kv_heads, head_dim, int(sliding), window)
    return out


def attention_decode_n(q, k_cache, v_cache, gate, n_cache, cap, q_heads, kv_heads, head_dim,
                       sliding=0, window=512):
    kc, vc = _as_f32_cache(k_cache), _as_f32_cache(v_cache)
    q = np.ascontiguousarray(q, np.float32)
    out = np.zeros((q_heads, head_dim), np.float32)
    g = None if gate is None else np.ascontiguousarray(gate, np.float32)
    lib().orc_attention_decode_n(_ptr(out), _ptr(q), _ptr(kc), _ptr(vc),
                                 None if g is None else _ptr(g), n_cache, cap, q_heads,
                                 kv_heads, head_dim, int(sliding), window)
    return out


def attention_prefill(q, k_cache, v_cache, gate, pos0, n_tok, cap, q_heads, kv_heads, head_dim,
                      sliding=0, window=512, t0=0, t1=None):
    kc, vc = _as_f32_cache(k_cache), _as_f32_cache(v_cache)
    q = np.ascontiguousarray(q, np.float32)
    out = np.zeros((n_tok, q_heads, head_dim), np.float32)
    g = None if gate is None else np.ascontiguousarray(gate, np.float32)
    lib().orc_attention_prefill(_ptr(out), _ptr(q), _ptr(kc), _ptr(vc),
                                None if g is None else _ptr(g), pos0, n_tok, cap, q_heads,
                                kv_heads, head_dim, int(sliding), window, t0,
                                n_tok if t1 is None else t1)
    return out


def payload_row_bytes(elems, group=64):
    return int(lib().orc_payload_row_bytes(elems, group))


def payload_encode_rows(rows: np.ndarray, group=64, variant=1) -> np.ndarray:
    rows = np.ascontiguousarray(rows, np.float32).reshape(-1, rows.shape[-1])
    elems = rows.shape[1]
    rb = payload_row_bytes(elems, group)
    out = np.empty((rows.shape[0], rb), np.uint8)
    for i in range(rows.shape[0]):
        lib().orc_payload_encode_row(_ptr(rows[i]), elems, group, variant, _ptr(out[i]))
    return out


def payload_decode_rows(enc: np.ndarray, elems, group=64) -> np.ndarray:
    enc = np.ascontiguousarray(enc, np.uint8).reshape(-1, payload_row_bytes(elems, group))
    out = np.empty((enc.shape[0], elems), np.float32)
    for i in range(enc.shape[0]):
        lib().orc_payload_decode_row(_ptr(enc[i]), elems, group, _ptr(out[i]))
    return out


def pack_layer(k_cache, v_cache, first_pos, rows, cap, kv_dim, fmt=0, group=64, variant=1):
    """KV section of one layer: fmt 0 raw f32 rows, fmt 1 int8-grouped payload."""
    eb = 4 if k_cache.dtype == np.float32 else 2
    rb = kv_dim * 4 if fmt == 0 else payload_row_bytes(kv_dim, group)
    out = np.empty(rows * 2 * rb, np.uint8)
    lib().orc_pack_layer(_ptr(out), _ptr(k_cache), _ptr(v_cache), eb, first_pos, rows, cap,
                         kv_dim, fmt, group, variant)
    return out


def unpack_layer(src, k_cache, v_cache, first_pos, rows, cap, kv_dim, fmt=0, group=64):
    eb = 4 if k_cache.dtype == np.float32 else 2
    src = np.ascontiguousarray(src, np.uint8)
    lib().orc_unpack_layer(_ptr(src), _ptr(k_cache), _ptr(v_cache), eb, first_pos, rows, cap,
                           kv_dim, fmt, group)


def qk_prep(x, w_bf16, rotary_dim, theta, llama3, pos, eps=1e-5):
    """RMS norm (weight w + 1) + split-half RoPE of heads x [..., 128] (copy)."""
    x = np.ascontiguousarray(x, np.float32).copy()
    w = np.ascontiguousarray(w_bf16, np.uint16)
    lib().orc_qk_prep(_ptr(x), x.size // x.shape[-1], x.shape[-1], _ptr(w), rotary_dim, theta, int(llama3),
                      pos, eps)
    return x


def q8_0_quantize(x):
    """(int8 codes [n], f32 scales [n/32]) of sf37_q8_0_quantize_activation."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    xq = np.zeros(((x.size + 31) // 32) * 32, np.int8)
    xs = np.zeros((x.size + 31) // 32, np.float32)
    lib().orc_q8_0_quantize(_ptr(x), _ptr(xq), _ptr(xs), x.size)
    return xq, xs


def q8_0_matvec(w, x, out_dim):
    """sf37_q8_0_matvec: w uint8 [out_dim][in_dim/32*34], x f32 [in_dim]."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    w = np.ascontiguousarray(w, np.uint8)
    out = np.zeros(out_dim, np.float32)
    lib().orc_q8_0_matvec(_ptr(out), _ptr(w), x.size, out_dim, _ptr(x))
    return out


def q8_0_abs_terms(w, x, out_dim):
    """sum_b |isum_b * wscale_b * xscale_b| per row: the magnitude a float
    accumulation error is relative to."""
    xq, xs = q8_0_quantize(x)
    nb = xs.size
    wb = np.asarray(w, np.uint8).reshape(out_dim, nb, 34)
    ws = wb[:, :, :2].copy().view(np.float16).reshape(out_dim, nb).astype(np.float64)
    wq = wb[:, :, 2:].view(np.int8).astype(np.int64)
    isum = (wq * xq.reshape(nb, 32).astype(np.int64)[None]).sum(-1)
    return np.abs(isum * ws * xs.astype(np.float64)[None]).sum(-1)


def bf16_bits_to_f32(w):
    return (np.asarray(w, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------- the reference's own CPU code
def ref_q8_0_quantize(x):
    R = ref()
    R.sf37_q8_0_quantize_activation.argtypes = [_vp, _vp, _vp, _u64]
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    xq = np.zeros(((x.size + 31) // 32) * 32, np.int8)
    xs = np.zeros((x.size + 31) // 32, np.float32)
    R.sf37_q8_0_quantize_activation(_ptr(x), _ptr(xq), _ptr(xs), x.size)
    return xq, xs


def ref_q8_0_matvec(w, x, out_dim):
    R = ref()
    R.sf37_q8_0_matvec.argtypes = [_vp, _vp, _u64, _u64, _vp]
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    w = np.ascontiguousarray(w, np.uint8)
    out = np.zeros(out_dim, np.float32)
    R.sf37_q8_0_matvec(_ptr(out), _ptr(w), x.size, out_dim, _ptr(x))
    return out


def ref_qk_prep(x, w_bf16, rotary_dim, theta, llama3, pos):
    """The reference's head_rms_norm_weight1 + apply_rope_one (copy of x)."""
    R = ref()
    R.sf37ref_qk_prep.argtypes = [_vp, _u32, _vp, _u32, ctypes.c_double, _int, _u32]
    x = np.ascontiguousarray(x, np.float32).copy()
    w = np.ascontiguousarray(bf16_bits_to_f32(w_bf16), np.float32)
    R.sf37ref_qk_prep(_ptr(x), x.size // 128, _ptr(w), rotary_dim, theta, int(llama3), pos)
    return x

def ref_payload_encode_rows(rows: np.ndarray, group=64) -> np.ndarray:
    rows = np.ascontiguousarray(rows, np.float32).reshape(-1, rows.shape[-1])
    R = ref()
    rb = int(R.sf37ref_payload_row_bytes(rows.shape[1], group))
    out = np.empty((rows.shape[0], rb), np.uint8)
    R.sf37ref_payload_encode_rows(_ptr(rows), rows.shape[1], group, rows.shape[0], _ptr(out))
    return out


def ref_payload_decode_rows(enc, elems, group=64):
    R = ref()
    rb = int(R.sf37ref_payload_row_bytes(elems, group))
    enc = np.ascontiguousarray(enc, np.uint8).reshape(-1, rb)
    out = np.empty((enc.shape[0], elems), np.float32)
    R.sf37ref_payload_decode_rows(_ptr(enc), elems, group, enc.shape[0], _ptr(out))
    return out


def ref_attention_decode(q, k_cache, v_cache, n_live, cap, q_heads, sliding, gate):
    """The reference CPU attention_decode (8 KV heads, head_dim 128, linear
    cache of n_live rows) followed by the sigmoid gate."""
    kc, vc = _as_f32_cache(k_cache), _as_f32_cache(v_cache)
    q = np.ascontiguousarray(q, np.float32)
    out = np.zeros((q_heads, 128), np.float32)
    g = None if gate is None else np.ascontiguousarray(gate, np.float32)
    ref().sf37ref_attention_decode(_ptr(out), _ptr(q), _ptr(kc), _ptr(vc), n_live, cap, q_heads,
                                   int(sliding), None if g is None else _ptr(g))
    return out


def ref_kv_cache_push(k_cache, v_cache, cap, n_live, k, v):
    """Reference kv_cache_push of len(k) rows; returns the new live count."""
    n = _u32(n_live)
    k = np.ascontiguousarray(k, np.float32).reshape(-1, 1024)
    v = np.ascontiguousarray(v, np.float32).reshape(-1, 1024)
    ref().sf37ref_kv_cache_push_rows(_ptr(k_cache), _ptr(v_cache), cap, ctypes.byref(n),
                                     _ptr(k), _ptr(v), k.shape[0])
    return n.value


# ------------------------------------------------ the reference's CUDA kernels
def ref_cuda_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libsf37ref_cuda.so"))


class RefTensor(ctypes.Structure):
    _fields_ = [("ptr", _vp), ("bytes", _u64)]


_refc = None


def ref_cuda():
    """The reference's own sf37_cuda.cu built for sm_100a (fp32 caches)."""
    global _refc
    if _refc is None:
        R = ctypes.CDLL(os.path.join(HERE, "_ref", "libsf37ref_cuda.so"))
        TP = ctypes.POINTER(RefTensor)
        R.sf37_cuda_init.restype = _int
        R.sf37_cuda_synchronize.restype = _int
        R.sf37_cuda_store_kv_cache_batch.restype = _int
        R.sf37_cuda_store_kv_cache_batch.argtypes = [TP] * 4 + [_u32] * 4
        for n in ("sf37_cuda_attention_decode_heads_at", "sf37_cuda_attention_decode_heads"):
            getattr(R, n).restype = _int
            getattr(R, n).argtypes = [TP] * 5 + [_u32] * 5 + [_int, _u32]
        R.sf37_cuda_attention_prefill_heads.restype = _int
        R.sf37_cuda_attention_prefill_heads.argtypes = [TP] * 5 + [_u32] * 6 + [_int, _u32]
        if not R.sf37_cuda_init():
            raise RuntimeError("reference sf37_cuda_init failed")
        _refc = R
    return _refc


def ref_tensor(ptr: int, nbytes: int):
    return ctypes.byref(RefTensor(ptr, nbytes))


# ---------------------------------------------------------------- cache sizing
def ref_sizing_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libsf37ref_sizing.so"))


_refs = None


def ref_sizing():
    """The reference engine's CUDA cache-sizing helpers (ref_sizing.c)."""
    global _refs
    if _refs is None:
        R = ctypes.CDLL(os.path.join(HERE, "_ref", "libsf37ref_sizing.so"))
        R.sf37ref_sliding_cache_cap.restype = _u32
        R.sf37ref_sliding_cache_cap.argtypes = [_u32, _u32]
        R.sf37ref_sliding_prefill_cap.restype = _u32
        R.sf37ref_sliding_prefill_cap.argtypes = [_u32, _u32]
        R.sf37ref_decode_kv_bytes_for_cap.restype = _u64
        R.sf37ref_decode_kv_bytes_for_cap.argtypes = [_u32]
        R.sf37ref_layer_is_full.restype = _int
        R.sf37ref_layer_is_full.argtypes = [_u32]
        _refs = R
    return _refs


def managed_kv_policy(kv_bytes, context_bytes, free_b, total_b):
    """sf37_cuda_should_use_managed_kv_cache (sf37_cuda.cu:1766-1800) on given
    free/total device bytes: 8 GiB KV or 8 GiB context thresholds, reserve
    total/4 clamped to [8, 40] GiB."""
    gib = 1 << 30
    if kv_bytes == 0:
        return 0
    if kv_bytes >= 8 * gib:
        return 1
    if context_bytes < 8 * gib:
        return 0
    reserve = min(max(total_b // 4, 8 * gib), 40 * gib)
    if context_bytes > free_b:
        return 1
    return int(free_b - context_bytes < reserve)
