"""CPU: sf37_kvstore record pieces that need no GPU -- the SHA-1 text key,
the 48-byte header writer and the header reader's rules -- against Python's
hashlib and the reference's own sf37_kvstore.c (oracle/_ref)."""
import ctypes
import hashlib

import numpy as np
import pytest

import oracle
from sf37_b200 import _lib

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def _sha(lib_fn, data):
    out = ctypes.create_string_buffer(41)
    buf = ctypes.create_string_buffer(bytes(data), len(data) or 1)
    lib_fn(buf, len(data), out)
    return out.value.decode()


@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 65, 119, 120, 1000, 1 << 20])
def test_sha1_matches_hashlib_and_reference(n):
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    got = _sha(_lib.lib().sf37kv_sha1_hex, data)
    assert got == hashlib.sha1(data).hexdigest()
    if oracle.ref_available():
        R = oracle.ref()
        R.sf37ref_sha1_hex.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p]
        assert got == _sha(R.sf37ref_sha1_hex, data)


@needs_ref
def test_header_bytes_match_reference():
    R = oracle.ref()
    args = [(37, 3, 1, 0, 4096, 0, 32768, 1700000000, 1700000123, 3423215356),
            (0, 8, 6, 0x1f, 1, 7, 262144, 0, 2 ** 64 - 1, 2 ** 40 + 5)]
    sig = [ctypes.c_void_p] + [ctypes.c_uint8] * 4 + [ctypes.c_uint32] * 3 + [ctypes.c_uint64] * 3
    R.sf37ref_kvstore_fill_header.argtypes = sig
    for a in args:
        mine = ctypes.create_string_buffer(48)
        ref = ctypes.create_string_buffer(48)
        _lib.lib().sf37kv_kvstore_fill_header(mine, *a)
        R.sf37ref_kvstore_fill_header(ref, *a)
        assert mine.raw == ref.raw


def test_header_reader_rules():
    # sf37_kvstore_read_header (sf37_kvstore.c:423-446): magic, version and
    # payload ABI must match; tokens != 0 and quant_bits == 3.
    L = _lib.lib()
    h = ctypes.create_string_buffer(52)
    L.sf37kv_kvstore_fill_header(h, 37, 3, 2, 1, 100, 4, 4096, 11, 22, 333)
    h[48:52] = (17).to_bytes(4, "little")
    e = _lib.KvstoreEntry()
    assert L.sf37kv_kvstore_parse_header(h, ctypes.byref(e)) == 1
    assert (e.model_id, e.quant_bits, e.reason, e.ext_flags, e.tokens, e.hits, e.ctx_size, e.created_at,
            e.last_used, e.payload_bytes, e.text_bytes) == (37, 3, 2, 1, 100, 4, 4096, 11, 22, 333, 17)
    for pos, val in ((0, ord("X")), (3, 2), (20, 1), (4, 8)):
        bad = ctypes.create_string_buffer(h.raw, 52)
        bad[pos] = val
        assert L.sf37kv_kvstore_parse_header(bad, ctypes.byref(e)) == 0, pos
    zero = ctypes.create_string_buffer(h.raw, 52)
    zero[8:12] = b"\0\0\0\0"
    assert L.sf37kv_kvstore_parse_header(zero, ctypes.byref(e)) == 0
    odd = ctypes.create_string_buffer(h.raw, 52)
    odd[5] = 9  # unknown reason codes read as 0 (unknown)
    assert L.sf37kv_kvstore_parse_header(odd, ctypes.byref(e)) == 1 and e.reason == 0
