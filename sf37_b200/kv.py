"""Torch-facing mirror of the KV-cache C ABI.

torch supplies device memory and streams only; every computation runs in
libsf37kv.so.  Function names and argument meaning follow the reference's
``sf37_cuda.h`` entry points (drop-in layer, fp32 caches, return True/False
like the reference's int 1/0) and ``include/sf37kv.h`` (native layer, raises
on error).
"""
import ctypes

import torch

from ._lib import AppendLayer, Cache, DecodeLayer, PackLayer, Tensor, check, lib

F16, F32 = 2, 4
Q_F32, Q_BF16 = 0, 1
FMT_RAW, FMT_I8G = 0, 1
_DT = {torch.float16: F16, torch.float32: F32}


def view(t):
    """sf37_cuda_tensor view {ptr, bytes} of a torch CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous()
    return ctypes.byref(Tensor(t.data_ptr(), t.numel() * t.element_size()))


def _sp(stream):
    if stream is None:
        return None
    return ctypes.c_void_p(stream.cuda_stream)


def _ptr(t):
    return None if t is None else t.data_ptr()


# ------------------------------------------------------------- drop-in layer
def store_kv_cache_batch(k_cache, v_cache, k, v, pos0, n_tok, cache_cap, kv_dim) -> bool:
    return bool(lib().sf37_cuda_store_kv_cache_batch(view(k_cache), view(v_cache), view(k), view(v),
                                                     pos0, n_tok, cache_cap, kv_dim))


def attention_decode_heads(out, q, k_cache, v_cache, gate, n_cache, cache_cap, q_heads, kv_heads,
                           head_dim, sliding, window) -> bool:
    return bool(lib().sf37_cuda_attention_decode_heads(view(out), view(q), view(k_cache),
                                                       view(v_cache), view(gate), n_cache,
                                                       cache_cap, q_heads, kv_heads, head_dim,
                                                       int(sliding), window))


def attention_decode_heads_at(out, q, k_cache, v_cache, gate, pos, cache_cap, q_heads, kv_heads,
                              head_dim, sliding, window) -> bool:
    return bool(lib().sf37_cuda_attention_decode_heads_at(view(out), view(q), view(k_cache),
                                                          view(v_cache), view(gate), pos, cache_cap,
                                                          q_heads, kv_heads, head_dim, int(sliding),
                                                          window))


def attention_prefill_heads(out, q, k_cache, v_cache, gate, pos0, n_tok, cache_cap, q_heads,
                            kv_heads, head_dim, sliding, window) -> bool:
    return bool(lib().sf37_cuda_attention_prefill_heads(view(out), view(q), view(k_cache),
                                                        view(v_cache), view(gate), pos0, n_tok,
                                                        cache_cap, q_heads, kv_heads, head_dim,
                                                        int(sliding), window))


def gqa_single_token_heads(out, v, gate, q_heads, kv_heads, head_dim) -> bool:
    return bool(lib().sf37_cuda_gqa_single_token_heads(view(out), view(v), view(gate), q_heads,
                                                       kv_heads, head_dim))


def kv_pack_rows(host_dst, k_cache, v_cache, first_pos, rows, cache_cap, kv_dim, fmt=FMT_RAW,
                 group=64, variant=1) -> bool:
    """sf37_cuda_kv_pack_rows_{f32,i8g}; host_dst: a writable numpy array."""
    p = host_dst.ctypes.data
    if fmt == FMT_RAW:
        return bool(lib().sf37_cuda_kv_pack_rows_f32(p, view(k_cache), view(v_cache), first_pos,
                                                     rows, cache_cap, kv_dim))
    return bool(lib().sf37_cuda_kv_pack_rows_i8g(p, view(k_cache), view(v_cache), first_pos, rows,
                                                 cache_cap, kv_dim, group, variant))


def kv_unpack_rows(host_src, k_cache, v_cache, first_pos, rows, cache_cap, kv_dim, fmt=FMT_RAW,
                   group=64) -> bool:
    p = host_src.ctypes.data
    if fmt == FMT_RAW:
        return bool(lib().sf37_cuda_kv_unpack_rows_f32(p, view(k_cache), view(v_cache), first_pos,
                                                       rows, cache_cap, kv_dim))
    return bool(lib().sf37_cuda_kv_unpack_rows_i8g(p, view(k_cache), view(v_cache), first_pos, rows,
                                                   cache_cap, kv_dim, group))


# ------------------------------------------------------------- native layer
def cache_desc(k_cache, v_cache, cap, sliding=False, window=512):
    return Cache(k_cache.data_ptr(), v_cache.data_ptr(), cap, int(bool(sliding)), window, 0)


def decode_layers_desc(layers):
    """layers: list of dicts with k_cache, v_cache, cap, sliding, window, pos, q, gate, out,
    k_new, v_new (tensors or None).  Returns a ctypes array (reusable)."""
    arr = (DecodeLayer * len(layers))()
    for i, L in enumerate(layers):
        arr[i] = DecodeLayer(cache_desc(L["k_cache"], L["v_cache"], L["cap"], L.get("sliding", 0),
                                        L.get("window", 512)), L["pos"], 0, _ptr(L["q"]),
                             _ptr(L.get("gate")), _ptr(L.get("out")), _ptr(L.get("k_new")),
                             _ptr(L.get("v_new")))
    return arr


def decode(layers, q_heads, kv_heads, head_dim, dtype, stream=None):
    arr = layers if not isinstance(layers, list) else decode_layers_desc(layers)
    check(lib().sf37kv_decode(arr, len(arr), q_heads, kv_heads, head_dim, dtype, _sp(stream)),
          "sf37kv_decode")


def qk_prep_desc(preps):
    """preps: list of dicts q_norm, k_norm (bf16 tensors as int16/uint16/bfloat16),
    rotary_dim, theta, llama3, eps.  Returns a ctypes array (reusable)."""
    from ._lib import QkPrep
    arr = (QkPrep * len(preps))()
    for i, p in enumerate(preps):
        arr[i] = QkPrep(_ptr(p["q_norm"]), _ptr(p.get("k_norm")), float(p["theta"]), int(p["rotary_dim"]),
                        int(p.get("llama3", 0)), float(p.get("eps", 1e-5)), 0)
    return arr


def decode_prep(layers, preps, q_heads, kv_heads, head_dim, dtype, stream=None):
    """sf37kv_decode with the q / k_new heads normalized and rotated in the kernel."""
    arr = layers if not isinstance(layers, list) else decode_layers_desc(layers)
    pa = preps if not isinstance(preps, list) else qk_prep_desc(preps)
    check(lib().sf37kv_decode_prep(arr, pa, len(arr), q_heads, kv_heads, head_dim, dtype, _sp(stream)),
          "sf37kv_decode_prep")


def append(layers, kv_dim, dtype, stream=None):
    arr = (AppendLayer * len(layers))()
    for i, L in enumerate(layers):
        arr[i] = AppendLayer(cache_desc(L["k_cache"], L["v_cache"], L["cap"]), L["pos0"], L["n_tok"],
                             _ptr(L["k"]), _ptr(L["v"]))
    check(lib().sf37kv_append(arr, len(arr), kv_dim, dtype, _sp(stream)), "sf37kv_append")


def prefill(k_cache, v_cache, cap, q, gate, out, pos0, n_tok, q_heads, kv_heads, head_dim, dtype,
            sliding=False, window=512, stream=None):
    c = cache_desc(k_cache, v_cache, cap, sliding, window)
    qt = Q_BF16 if q.dtype == torch.bfloat16 else Q_F32
    check(lib().sf37kv_prefill(ctypes.byref(c), _ptr(q), qt, _ptr(gate), _ptr(out), pos0, n_tok,
                               q_heads, kv_heads, head_dim, dtype, _sp(stream)), "sf37kv_prefill")


def row_bytes(kv_dim, fmt, group=64) -> int:
    return int(lib().sf37kv_row_bytes(kv_dim, fmt, group))


def pack_layers_desc(layers, kv_dim, fmt, group=64):
    """layers: list of dicts with k_cache, v_cache, cap, first_pos, rows.  Sections are laid
    out back to back; returns (ctypes array, total bytes)."""
    arr = (PackLayer * len(layers))()
    rb = row_bytes(kv_dim, fmt, group)
    off = 0
    for i, L in enumerate(layers):
        arr[i] = PackLayer(cache_desc(L["k_cache"], L["v_cache"], L["cap"]), L["first_pos"],
                           L["rows"], off)
        off += 2 * L["rows"] * rb
    return arr, off


def pack(dst, arr, kv_dim, dtype, fmt, group=64, variant=1, stream=None):
    """dst: torch CUDA uint8 tensor (or an int device/mapped-host address)."""
    p = dst if isinstance(dst, int) else dst.data_ptr()
    check(lib().sf37kv_pack(p, arr, len(arr), kv_dim, dtype, fmt, group, variant, _sp(stream)),
          "sf37kv_pack")


def unpack(src, arr, kv_dim, dtype, fmt, group=64, stream=None):
    p = src if isinstance(src, int) else src.data_ptr()
    check(lib().sf37kv_unpack(p, arr, len(arr), kv_dim, dtype, fmt, group, _sp(stream)),
          "sf37kv_unpack")


def pack_to_host(host_ptr, arr, kv_dim, dtype, fmt, group=64, variant=1):
    check(lib().sf37kv_pack_to_host(host_ptr, arr, len(arr), kv_dim, dtype, fmt, group, variant),
          "sf37kv_pack_to_host")


def unpack_from_host(host_ptr, arr, kv_dim, dtype, fmt, group=64):
    check(lib().sf37kv_unpack_from_host(host_ptr, arr, len(arr), kv_dim, dtype, fmt, group),
          "sf37kv_unpack_from_host")


def set_stream(stream):
    lib().sf37kv_set_stream(_sp(stream))


def launch_count() -> int:
    return int(lib().sf37kv_launch_count())


def device_error(clear=False) -> int:
    """The device error flag (0 = none, 2 = a bounded wait timed out); syncs."""
    return lib().sf37kv_device_error(int(bool(clear)))


def oproj(layers, in_dim, out_dim, stream=None):
    """Q8_0 o_proj matvec of every layer in one launch (sf37kv_oproj_q8_0)."""
    check(lib().sf37kv_oproj_q8_0(layers, len(layers), in_dim, out_dim, _sp(stream)), "sf37kv_oproj_q8_0")
