"""sf37_b200: the SF37 KV-cache hot path on B200 (sm_100a).

The product is the C ABI library ``libsf37kv.so`` (declared in ``include/``):
drop-in replacements for the reference's ``sf37_cuda.h`` KV entry points and
a native f16 / multi-layer / streamed API.  This package builds it
(``sf37_b200.build``), binds it with ctypes (``sf37_b200._lib``) and offers a
thin torch-facing mirror of the reference interface (``sf37_b200.kv``).
"""
from ._lib import lib, last_error, LIB_PATH  # noqa: F401
