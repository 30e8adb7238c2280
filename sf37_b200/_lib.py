"""ctypes binding of libsf37kv.so (the C ABI declared in include/*.h).

There is no fallback: if the shared library is missing or fails to load,
every call raises.  Build it with ``python -m sf37_b200.build``.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsf37kv.so")

c_u32, c_u64, c_int, c_vp, c_float = (ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int,
                                      ctypes.c_void_p, ctypes.c_float)


class Tensor(ctypes.Structure):
    """struct sf37_cuda_tensor {void *ptr; uint64_t bytes;} (sf37_cuda.cu:32-35)."""
    _fields_ = [("ptr", c_vp), ("bytes", c_u64)]


class Cache(ctypes.Structure):
    _fields_ = [("k_cache", c_vp), ("v_cache", c_vp), ("cap", c_u32), ("sliding", c_u32),
                ("window", c_u32), ("reserved", c_u32)]


class DecodeLayer(ctypes.Structure):
    _fields_ = [("cache", Cache), ("pos", c_u32), ("reserved", c_u32), ("q", c_vp),
                ("gate", c_vp), ("out", c_vp), ("k_new", c_vp), ("v_new", c_vp)]


class AppendLayer(ctypes.Structure):
    _fields_ = [("cache", Cache), ("pos0", c_u32), ("n_tok", c_u32), ("k", c_vp), ("v", c_vp)]


class PeerGather(ctypes.Structure):
    _fields_ = [("peer_buf", c_vp * 8), ("peer_flags", c_vp * 8), ("my_flags", c_vp),
                ("done_counter", c_vp), ("world", c_u32), ("rank", c_u32)]


class QkPrep(ctypes.Structure):
    _fields_ = [("q_norm", c_vp), ("k_norm", c_vp), ("theta", ctypes.c_double), ("rotary_dim", c_u32),
                ("llama3", c_u32), ("eps", c_float), ("reserved", c_u32)]


class OprojLayer(ctypes.Structure):
    _fields_ = [("weights", c_vp), ("x", c_vp), ("out", c_vp)]


class PackLayer(ctypes.Structure):
    _fields_ = [("cache", Cache), ("first_pos", c_u32), ("rows", c_u32), ("offset", c_u64)]


class SessionLayout(ctypes.Structure):
    _fields_ = [("n_layers", c_u32), ("kv_heads", c_u32), ("head_dim", c_u32), ("vocab", c_u32),
                ("embd", c_u32), ("sliding_window", c_u32), ("full_every", c_u32),
                ("payload_group", c_u32)]


class Session(ctypes.Structure):
    _fields_ = [("layout", SessionLayout), ("ctx_size", ctypes.c_int32), ("n_tokens", c_u32),
                ("tokens", c_vp), ("logits", c_vp), ("hidden", c_vp), ("caches", ctypes.POINTER(Cache)),
                ("dtype", c_int), ("backend_kind", c_u32)]


class KvstoreEntry(ctypes.Structure):
    _fields_ = [("quant_bits", ctypes.c_uint8), ("model_id", ctypes.c_uint8), ("reason", ctypes.c_uint8),
                ("ext_flags", ctypes.c_uint8), ("tokens", c_u32), ("hits", c_u32), ("ctx_size", c_u32),
                ("text_bytes", c_u32), ("created_at", c_u64), ("last_used", c_u64), ("payload_bytes", c_u64)]


class CachePlan(ctypes.Structure):
    _fields_ = [("ctx_size", c_u32), ("window", c_u32), ("sliding_cap", c_u32), ("prefill_cap", c_u32),
                ("full_layers", c_u32), ("sliding_layers", c_u32), ("cap", c_u32 * 64), ("sliding", c_u32 * 64),
                ("kv_cache_bytes", c_u64)]


TP = ctypes.POINTER(Tensor)
SP = ctypes.POINTER(Session)

# name -> (restype, argtypes); every symbol include/*.h declares.
SIGNATURES = {
    # include/sf37_cuda_kv.h
    "sf37_cuda_device_count": (c_int, []),
    "sf37_cuda_init": (c_int, []),
    "sf37_cuda_cleanup": (None, []),
    "sf37_cuda_synchronize": (c_int, []),
    "sf37_cuda_memory_info": (c_int, [ctypes.POINTER(c_u64), ctypes.POINTER(c_u64)]),
    "sf37_cuda_tensor_alloc": (TP, [c_u64]),
    "sf37_cuda_tensor_alloc_managed": (TP, [c_u64]),
    "sf37_cuda_tensor_free": (None, [TP]),
    "sf37_cuda_tensor_bytes": (c_u64, [TP]),
    "sf37_cuda_tensor_write": (c_int, [TP, c_u64, c_vp, c_u64]),
    "sf37_cuda_tensor_read": (c_int, [TP, c_u64, c_vp, c_u64]),
    "sf37_cuda_tensor_copy": (c_int, [TP, c_u64, TP, c_u64, c_u64]),
    "sf37_cuda_tensor_fill_f32": (c_int, [TP, c_float, c_u64]),
    "sf37_cuda_gqa_single_token_heads": (c_int, [TP, TP, TP, c_u32, c_u32, c_u32]),
    "sf37_cuda_attention_decode_heads": (c_int, [TP] * 5 + [c_u32] * 5 + [c_int, c_u32]),
    "sf37_cuda_attention_decode_heads_at": (c_int, [TP] * 5 + [c_u32] * 5 + [c_int, c_u32]),
    "sf37_cuda_matvec_q8_0": (c_int, [TP, TP, c_u64, c_u64, TP]),
    "sf37_cuda_should_use_managed_kv_cache": (c_int, [c_u64, c_u64]),
    "sf37_cuda_store_kv_cache_batch": (c_int, [TP] * 4 + [c_u32] * 4),
    "sf37_cuda_attention_prefill_heads": (c_int, [TP] * 5 + [c_u32] * 6 + [c_int, c_u32]),
    "sf37_cuda_kv_pack_rows_f32": (c_int, [c_vp, TP, TP, c_u32, c_u32, c_u32, c_u32]),
    "sf37_cuda_kv_unpack_rows_f32": (c_int, [c_vp, TP, TP, c_u32, c_u32, c_u32, c_u32]),
    "sf37_cuda_kv_pack_rows_i8g": (c_int, [c_vp, TP, TP] + [c_u32] * 5 + [c_int]),
    "sf37_cuda_kv_unpack_rows_i8g": (c_int, [c_vp, TP, TP] + [c_u32] * 5),
    # include/sf37kv.h
    "sf37kv_last_error": (ctypes.c_char_p, []),
    "sf37kv_version": (ctypes.c_char_p, []),
    "sf37kv_set_stream": (c_int, [c_vp]),
    "sf37kv_get_stream": (c_vp, []),
    "sf37kv_decode": (c_int, [ctypes.POINTER(DecodeLayer), c_u32, c_u32, c_u32, c_u32, c_int, c_vp]),
    "sf37kv_decode_noalloc": (c_int, [ctypes.POINTER(DecodeLayer), c_u32, c_u32, c_u32, c_u32, c_int,
                                      c_vp]),
    "sf37kv_append": (c_int, [ctypes.POINTER(AppendLayer), c_u32, c_u32, c_int, c_vp]),
    "sf37kv_prefill": (c_int, [ctypes.POINTER(Cache), c_vp, c_int, c_vp, c_vp, c_u32, c_u32,
                               c_u32, c_u32, c_u32, c_int, c_vp]),
    "sf37kv_row_bytes": (c_u64, [c_u32, c_int, c_u32]),
    "sf37kv_pack": (c_int, [c_vp, ctypes.POINTER(PackLayer), c_u32, c_u32, c_int, c_int, c_u32,
                            c_int, c_vp]),
    "sf37kv_unpack": (c_int, [c_vp, ctypes.POINTER(PackLayer), c_u32, c_u32, c_int, c_int, c_u32,
                              c_vp]),
    "sf37kv_host_alloc": (c_vp, [c_u64]),
    "sf37kv_host_free": (None, [c_vp]),
    "sf37kv_pack_to_host": (c_int, [c_vp, ctypes.POINTER(PackLayer), c_u32, c_u32, c_int, c_int,
                                    c_u32, c_int]),
    "sf37kv_unpack_from_host": (c_int, [c_vp, ctypes.POINTER(PackLayer), c_u32, c_u32, c_int,
                                        c_int, c_u32]),
    "sf37kv_launch_count": (c_u64, []),
    "sf37kv_device_error": (c_int, [c_int]),
    "sf37kv_dev_alloc": (c_vp, [c_u64]),
    "sf37kv_dev_free": (None, [c_vp]),
    "sf37kv_ipc_handle": (c_int, [c_vp, c_vp]),
    "sf37kv_ipc_open": (c_vp, [c_vp]),
    "sf37kv_ipc_close": (None, [c_vp]),
    "sf37kv_decode_prep": (c_int, [ctypes.POINTER(DecodeLayer), ctypes.POINTER(QkPrep), c_u32, c_u32, c_u32,
                                   c_u32, c_int, c_vp]),
    "sf37kv_pack_slice_to_host": (c_int, [c_vp, ctypes.POINTER(PackLayer), c_u32, c_u32, c_u32, c_u32, c_int,
                                          c_int, c_u32, c_int]),
    "sf37kv_unpack_slice_from_host": (c_int, [c_vp, ctypes.POINTER(PackLayer), c_u32, c_u32, c_u32, c_u32, c_int,
                                              c_int, c_u32]),
    "sf37kv_oproj_q8_0": (c_int, [ctypes.POINTER(OprojLayer), c_u32, c_u32, c_u32, c_vp]),
    "sf37kv_oproj_q8_0_shard": (c_int, [ctypes.POINTER(OprojLayer), c_u32, c_u32, c_u32, c_u64,
                                        ctypes.POINTER(PeerGather), c_u32, c_vp]),
    "sf37kv_oproj_reduce": (c_int, [ctypes.POINTER(PeerGather), c_u32, c_u32, c_u32, c_vp, c_vp]),
    "sf37kv_q8_0_quantize": (c_int, [c_vp, c_vp, c_vp, c_u64, c_vp]),
    "sf37kv_decode_gather": (c_int, [ctypes.POINTER(DecodeLayer), c_u32, c_u32, c_u32, c_u32, c_int,
                                     ctypes.POINTER(PeerGather), c_u32, c_vp]),
    "sf37kv_gather_wait": (c_int, [ctypes.POINTER(PeerGather), c_u32, c_vp]),
    "sf37kv_sliding_cache_cap": (c_u32, [c_u32, c_u32]),
    "sf37kv_sliding_prefill_cap": (c_u32, [c_u32, c_u32]),
    "sf37kv_kv_cache_bytes": (c_u64, [c_u32, c_u32, c_u32, c_int]),
    "sf37kv_prefill_default_chunk": (c_u32, [c_u64]),
    "sf37kv_plan_caches": (c_int, [c_u32, c_u32, c_u32, c_u32, c_u32, c_int, ctypes.POINTER(CachePlan)]),
    "sf37kv_managed_kv_policy": (c_int, [c_u64, c_u64, c_u64, c_u64]),
    # include/sf37kv_session.h
    "sf37kv_session_layout_default": (SessionLayout, []),
    "sf37kv_session_snapshot_bytes": (c_u64, [SP]),
    "sf37kv_session_payload_bytes": (c_u64, [SP]),
    "sf37kv_session_save_snapshot": (c_int, [SP, c_vp, c_u64, ctypes.POINTER(c_u64), ctypes.c_char_p,
                                             ctypes.c_size_t]),
    "sf37kv_session_load_snapshot": (c_int, [SP, c_vp, c_u64, ctypes.c_char_p, ctypes.c_size_t]),
    "sf37kv_session_save_payload": (c_int, [SP, c_int, ctypes.c_char_p, ctypes.c_size_t]),
    "sf37kv_session_load_payload": (c_int, [SP, c_int, c_u64, ctypes.c_char_p, ctypes.c_size_t]),
    "sf37kv_kvstore_fill_header": (None, [c_vp, ctypes.c_uint8, ctypes.c_uint8, ctypes.c_uint8, ctypes.c_uint8,
                                          c_u32, c_u32, c_u32, c_u64, c_u64, c_u64]),
    "sf37kv_kvstore_parse_header": (c_int, [c_vp, ctypes.POINTER(KvstoreEntry)]),
    "sf37kv_sha1_hex": (None, [c_vp, ctypes.c_size_t, ctypes.c_char_p]),
    "sf37kv_kvstore_save": (c_int, [SP, c_int, ctypes.c_char_p, c_u32, ctypes.c_uint8, ctypes.c_uint8, c_u64,
                                    ctypes.POINTER(c_u64), ctypes.c_char_p, ctypes.c_size_t]),
    "sf37kv_kvstore_load": (c_int, [SP, c_int, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p,
                                    ctypes.POINTER(c_u32), ctypes.c_char_p, ctypes.c_size_t]),
}

_lib = None


def lib():
    """Loads libsf37kv.so (raising if it is absent) and binds SIGNATURES."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m sf37_b200.build` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().sf37kv_last_error().decode()


def check(rc: int, what: str):
    """Raises on a nonzero native status code."""
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {last_error()}")
