"""Batched RWKV-7 decode handle over the C ABI (sn_abi_rwkv7_*_batch).

One handle owns `nseq` sequences, each with its (L, NH, HS, HS) matrix state
and (L, 2, D) token shift in HBM. Loads KRWK v3 (fp32 / INT4 block 64) and
KRWK v4 (INT4 group G, fp16 scales) blobs.
"""
from __future__ import annotations

import numpy as np

from . import _lib
from ._lib import check, ptr
from .model import _out_like, _tokens
from .runtime import bind_stream, load_runtime


class Rwkv7Batch:
    def __init__(self, path, nseq: int = 1):
        self._lib = load_runtime()
        self._h = self._lib.sn_abi_rwkv7_load_batch(str(path).encode(), int(nseq))
        if not self._h:
            raise RuntimeError(f"sn_abi_rwkv7_load_batch failed: {_lib.last_error()}")
        d = np.zeros(8, np.int32)
        self._lib.sn_abi_rwkv7_dims(self._h, ptr(d))
        self.vocab, self.dim, self.head_size, self.n_head, self.ffn, self.layers, self.q4, \
            self.group = (int(v) for v in d)
        self.nseq = int(nseq)

    def step(self, tokens, logits=None):
        t = _tokens(tokens)
        B = int(t.shape[0])
        if logits is None:
            logits = _out_like(t, (B, self.vocab), np.float32)
        bind_stream(t, logits)
        check(self._lib.sn_abi_rwkv7_step_batch(self._h, ptr(t), B, ptr(logits)), "rwkv7_step")
        return logits

    def step_argmax(self, tokens, out=None):
        t = _tokens(tokens)
        B = int(t.shape[0])
        if out is None:
            out = _out_like(t, (B,), np.int32)
        bind_stream(t, out)
        check(self._lib.sn_abi_rwkv7_step_argmax(self._h, ptr(t), B, ptr(out)), "rwkv7_argmax")
        return out

    def prefill(self, tokens, logits=None, want_logits: bool = True):
        """tokens (B, T) -> logits (B, vocab) of each sequence's last token:
        every layer over all prompt rows at once, the recurrence in order."""
        if hasattr(tokens, "data_ptr"):
            import torch
            t = tokens.to(torch.int32).contiguous()
        else:
            t = np.ascontiguousarray(np.asarray(tokens, np.int32))
        B, T = t.shape
        if want_logits and logits is None:
            logits = _out_like(t, (B, self.vocab), np.float32)
        bind_stream(t, logits)
        check(self._lib.sn_abi_rwkv7_prefill_batch(self._h, ptr(t), B, T,
                                                   ptr(logits) if want_logits else None),
              "rwkv7_prefill")
        return logits

    def step_trace(self, tokens):
        """One step that also returns the residual stream entering each layer
        and leaving the last: (logits (B, vocab), xs (B, L+1, D)), host arrays."""
        t = np.ascontiguousarray(np.asarray(tokens, np.int32))
        B = int(t.shape[0])
        logits = np.empty((B, self.vocab), np.float32)
        xs = np.empty((B, self.layers + 1, self.dim), np.float32)
        check(self._lib.sn_abi_rwkv7_step_trace(self._h, ptr(t), B, ptr(logits), ptr(xs)),
              "rwkv7_step_trace")
        return logits, xs

    def reset(self):
        check(self._lib.sn_abi_rwkv7_reset(self._h), "rwkv7_reset")

    def get_state(self, B=None):
        B = self.nseq if B is None else B
        S = np.empty((B, self.layers, self.n_head, self.head_size, self.head_size), np.float32)
        sh = np.empty((B, self.layers, 2, self.dim), np.float32)
        check(self._lib.sn_abi_rwkv7_get_state(self._h, B, ptr(S), ptr(sh)), "rwkv7_state")
        return S, sh

    def close(self):
        if getattr(self, "_h", None):
            self._lib.sn_abi_rwkv7_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
