"""Session KV checkpoints (include/sf37kv_session.h) for torch-held caches.

Mirrors the reference's sf37_session_* checkpoint calls (sf37.h:153-164;
sf37.c:6809-7500): save_snapshot / load_snapshot (raw format 2, in memory),
save_payload / load_payload (int8-grouped format 3, on a file descriptor).
A failure raises SessionError carrying the reference's message.
"""
import ctypes
import os

import numpy as np
import torch

from ._lib import Cache, Session as _Session, lib
from .kv import F16, F32


class SessionError(RuntimeError):
    pass


def default_layout():
    return lib().sf37kv_session_layout_default()


class Session:
    """Checkpoint state of one sequence: ctx_size, tokens, logits, hidden and
    the device KV caches, one (k, v) pair of [cap][kv_heads*head_dim] torch
    tensors (f32 or f16) per layer; position p lives in slot p % cap."""

    def __init__(self, ctx_size, caches, layout=None, backend_kind=1):
        self.layout = layout or default_layout()
        if len(caches) != self.layout.n_layers:
            raise ValueError(f"{len(caches)} caches for a {self.layout.n_layers}-layer layout")
        self.ctx_size = int(ctx_size)
        self.caches = caches
        dt = caches[0][0].dtype
        if dt not in (torch.float32, torch.float16):
            raise ValueError("caches must be float32 or float16")
        self.dtype = F32 if dt == torch.float32 else F16
        self.backend_kind = backend_kind
        self.tokens = np.zeros(max(self.ctx_size, 1), np.int32)
        self.n_tokens = 0
        self.logits = np.zeros(self.layout.vocab, np.float32)
        self.hidden = np.zeros(self.layout.embd, np.float32)
        self._cache_arr = (Cache * len(caches))()
        for i, (k, v) in enumerate(caches):
            if k.dtype != dt or v.dtype != dt or k.shape != v.shape:
                raise ValueError(f"layer {i}: k and v must share dtype and shape")
            self._cache_arr[i] = Cache(k.data_ptr(), v.data_ptr(), k.shape[0], 0, 0, 0)

    def set_tokens(self, tokens):
        t = np.asarray(tokens, np.int32)
        if t.size > self.tokens.size:
            self.tokens = np.zeros(t.size, np.int32)
        self.tokens[:t.size] = t
        self.n_tokens = int(t.size)

    def _struct(self):
        s = _Session()
        s.layout = self.layout
        s.ctx_size = self.ctx_size
        s.n_tokens = self.n_tokens
        s.tokens = self.tokens.ctypes.data
        s.logits = self.logits.ctypes.data
        s.hidden = self.hidden.ctypes.data
        s.caches = self._cache_arr
        s.dtype = self.dtype
        s.backend_kind = self.backend_kind
        return s

    def _sync_in(self):
        # the library reads the caches on its stream; finish torch's writes
        torch.cuda.synchronize()

    def snapshot_bytes(self) -> int:
        return int(lib().sf37kv_session_snapshot_bytes(ctypes.byref(self._struct())))

    def payload_bytes(self) -> int:
        return int(lib().sf37kv_session_payload_bytes(ctypes.byref(self._struct())))

    def save_snapshot(self, out=None) -> torch.Tensor:
        """Raw snapshot into `out` (a uint8 CPU tensor, pinned for speed) or a
        new pinned buffer; returns the filled uint8 view."""
        n = self.snapshot_bytes()
        if out is None:
            out = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        if out.numel() < n:
            raise SessionError("session snapshot writer overflow")
        self._sync_in()
        err = ctypes.create_string_buffer(512)
        ln = ctypes.c_uint64(0)
        if lib().sf37kv_session_save_snapshot(ctypes.byref(self._struct()), out.data_ptr(), out.numel(),
                                              ctypes.byref(ln), err, 512):
            raise SessionError(err.value.decode())
        return out[:ln.value]

    def load_snapshot(self, buf):
        """Restores a raw snapshot (bytes, numpy uint8 or a CPU uint8 tensor)."""
        if isinstance(buf, torch.Tensor):
            ptr, n, keep = buf.data_ptr(), buf.numel(), buf
        else:
            keep = np.frombuffer(buf, np.uint8) if isinstance(buf, (bytes, bytearray)) else np.asarray(buf)
            ptr, n = keep.ctypes.data, keep.size
        self._sync_in()
        s = self._struct()
        err = ctypes.create_string_buffer(512)
        if lib().sf37kv_session_load_snapshot(ctypes.byref(s), ptr, n, err, 512):
            raise SessionError(err.value.decode())
        del keep
        self.n_tokens = s.n_tokens

    def save_payload(self, f):
        """Payload to a file object or descriptor at its current offset;
        returns the bytes written."""
        fd = f if isinstance(f, int) else f.fileno()
        if not isinstance(f, int):
            f.flush()
        self._sync_in()
        start = os.lseek(fd, 0, os.SEEK_CUR)
        err = ctypes.create_string_buffer(512)
        if lib().sf37kv_session_save_payload(ctypes.byref(self._struct()), fd, err, 512):
            raise SessionError(err.value.decode())
        return os.lseek(fd, 0, os.SEEK_CUR) - start

    def load_payload(self, f, nbytes):
        fd = f if isinstance(f, int) else f.fileno()
        self._sync_in()
        s = self._struct()
        err = ctypes.create_string_buffer(512)
        if lib().sf37kv_session_load_payload(ctypes.byref(s), fd, nbytes, err, 512):
            raise SessionError(err.value.decode())
        self.n_tokens = s.n_tokens

    def kvstore_save(self, f, text, reason=1, ext_flags=0, now=None):
        """An sf37_kvstore record (header, text, payload) to a file object or
        descriptor at its current offset; returns the record's bytes."""
        import time as _time
        fd = f if isinstance(f, int) else f.fileno()
        if not isinstance(f, int):
            f.flush()
        self._sync_in()
        tb = text.encode() if isinstance(text, str) else bytes(text)
        n = ctypes.c_uint64(0)
        err = ctypes.create_string_buffer(512)
        now = int(_time.time()) if now is None else int(now)
        if lib().sf37kv_kvstore_save(ctypes.byref(self._struct()), fd, tb, len(tb), reason, ext_flags, now,
                                     ctypes.byref(n), err, 512):
            raise SessionError(err.value.decode())
        return n.value

    def kvstore_load(self, f, prompt, sha=None):
        """Restores a record whose text is a byte prefix of prompt; returns
        the tokens restored (raises SessionError with the reference's
        message otherwise)."""
        fd = f if isinstance(f, int) else f.fileno()
        self._sync_in()
        s = self._struct()
        pb = prompt.encode() if isinstance(prompt, str) else bytes(prompt)
        got = ctypes.c_uint32(0)
        err = ctypes.create_string_buffer(512)
        if lib().sf37kv_kvstore_load(ctypes.byref(s), fd, pb, len(pb), None if sha is None else sha.encode(),
                                     ctypes.byref(got), err, 512):
            raise SessionError(err.value.decode())
        self.n_tokens = s.n_tokens
        return got.value
