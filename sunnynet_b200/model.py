"""Batched SunnyNet decode handle over the C ABI (sn_abi_sunny_*).

One handle owns `nseq` independent sequences (weights and state in HBM). A
step feeds one token to each of the first B sequences and returns logits
(B, vocab), or only the greedy next tokens. Arrays may be numpy (host) or
torch (host or CUDA) -- CUDA tensors avoid host copies.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import check, ptr
from .runtime import bind_stream, load_runtime


def _out_like(tokens, shape, dtype):
    if hasattr(tokens, "data_ptr"):
        import torch
        return torch.empty(shape, dtype={np.float32: torch.float32, np.int32: torch.int32}[dtype],
                           device=tokens.device)
    return np.empty(shape, dtype)


def _tokens(t):
    if hasattr(t, "data_ptr"):
        import torch
        return t.to(torch.int32).contiguous()
    return np.ascontiguousarray(np.asarray(t, np.int32).reshape(-1))


class SunnyBatch:
    def __init__(self, path, nseq: int = 1):
        self._lib = load_runtime()
        self._h = self._lib.sn_abi_sunny_load(str(path).encode(), int(nseq))
        if not self._h:
            raise RuntimeError(f"sn_abi_sunny_load failed: {_lib.last_error()}")
        d = np.zeros(8, np.int32)
        self._lib.sn_abi_sunny_dims(self._h, ptr(d))
        self.vocab, self.dim, self.inner, self.rank, self.taps, self.layers, self.group, \
            self.wtype = (int(v) for v in d)
        self.nseq = int(nseq)

    def step(self, tokens, logits=None):
        t = _tokens(tokens)
        B = int(t.shape[0])
        if logits is None:
            logits = _out_like(t, (B, self.vocab), np.float32)
        bind_stream(t, logits)
        check(self._lib.sn_abi_sunny_step(self._h, ptr(t), B, ptr(logits)), "sunny_step")
        return logits

    def step_argmax(self, tokens, out=None):
        t = _tokens(tokens)
        B = int(t.shape[0])
        if out is None:
            out = _out_like(t, (B,), np.int32)
        bind_stream(t, out)
        check(self._lib.sn_abi_sunny_step_argmax(self._h, ptr(t), B, ptr(out)), "sunny_argmax")
        return out

    def prefill(self, tokens, chunk: int = 256, logits=None, want_logits: bool = True):
        """tokens (B, T) -> logits of the last position (B, vocab). Runs as
        `chunk`-token chunks carrying only the recurrent state."""
        if hasattr(tokens, "data_ptr"):
            import torch
            t = tokens.to(torch.int32).contiguous()
        else:
            t = np.ascontiguousarray(np.asarray(tokens, np.int32))
        B, T = t.shape
        if want_logits and logits is None:
            logits = _out_like(t, (B, self.vocab), np.float32)
        bind_stream(t, logits)
        check(self._lib.sn_abi_sunny_prefill_chunked(self._h, ptr(t), B, T, int(chunk),
                                                     ptr(logits) if want_logits else None),
              "sunny_prefill")
        return logits

    def reset(self):
        check(self._lib.sn_abi_sunny_reset(self._h), "sunny_reset")

    def get_state(self, B=None):
        B = self.nseq if B is None else B
        kh = max(self.taps - 1, 1)
        s = np.empty((B, self.layers, self.dim), np.float32)
        h = np.empty((B, self.layers, kh, self.dim), np.float32)
        check(self._lib.sn_abi_sunny_get_state(self._h, B, ptr(s), ptr(h)), "get_state")
        return s, h

    def set_state(self, s, h):
        s = np.ascontiguousarray(s, np.float32)
        h = np.ascontiguousarray(h, np.float32)
        check(self._lib.sn_abi_sunny_set_state(self._h, s.shape[0], ptr(s), ptr(h)), "set_state")

    def get_state_at(self, seq0: int, n: int, s=None, h=None):
        """State of sequences [seq0, seq0+n) into s (n,L,D), h (n,L,K-1,D):
        numpy arrays, or CUDA tensors (then copied device to device)."""
        kh = max(self.taps - 1, 1)
        if s is None:
            s = np.empty((n, self.layers, self.dim), np.float32)
            h = np.empty((n, self.layers, kh, self.dim), np.float32)
        check(self._lib.sn_abi_sunny_get_state_at(self._h, int(seq0), int(n), ptr(s), ptr(h)),
              "get_state_at")
        return s, h

    def set_state_at(self, seq0: int, s, h):
        """Overwrite the state of sequences [seq0, seq0 + len(s))."""
        if not hasattr(s, "data_ptr"):
            s = np.ascontiguousarray(s, np.float32)
            h = np.ascontiguousarray(h, np.float32)
        check(self._lib.sn_abi_sunny_set_state_at(self._h, int(seq0), int(s.shape[0]), ptr(s),
                                                  ptr(h)), "set_state_at")

    def reset_at(self, seq0: int, n: int = 1):
        check(self._lib.sn_abi_sunny_reset_at(self._h, int(seq0), int(n)), "reset_at")

    def close(self):
        if getattr(self, "_h", None):
            self._lib.sn_abi_sunny_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
