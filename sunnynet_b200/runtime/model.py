"""B=1 SunnyNet handle over the reference's internal ABI (sunnynet.h), on a B200.

Same class and functions as the reference's ``sunnynet/runtime/model.py``
(``SnModel``, ``set_threads``, ``get_threads``, ``recommended_threads``), so the
CLI's ``--backend`` hook can construct either. Weights and state live in HBM.
"""
from __future__ import annotations

import ctypes

from .. import _lib
from . import load_runtime

__all__ = ["SnModel", "model_available", "set_threads", "get_threads", "recommended_threads"]


def model_available() -> bool:
    return _lib.LIB_PATH.exists()


def set_threads(n: int) -> int:
    lib = load_runtime()
    lib.sn_set_threads(int(n))
    return lib.sn_get_threads()


def get_threads() -> int:
    return load_runtime().sn_get_threads()


def recommended_threads() -> int:
    n = int(load_runtime().sn_recommended_threads())
    if n <= 0:
        import os
        n = max(1, (os.cpu_count() or 2) // 2)
    return n


class SnModel:
    """B=1 decode handle; logits reuse one host buffer (runtime/model.py:290-326)."""

    def __init__(self, path, vocab, dim, inner, rank, taps, layers, group=8, tied=1, half=False):
        self._lib = load_runtime()
        self._logits = (ctypes.c_float * vocab)()
        load = self._lib.sn_load_h if half else self._lib.sn_load
        self._h = load(str(path).encode(), vocab, dim, inner, rank, taps, layers, group, int(tied))
        if not self._h:
            raise RuntimeError(f"sn_load failed: {path} ({_lib.last_error()})")
        if not self._lib.sn_ready(self._h):
            raise RuntimeError("sn_load returned a handle that is not ready")
        self.vocab = vocab

    def reset(self):
        self._lib.sn_reset(self._h)

    def step(self, token: int) -> list:
        self._lib.sn_step(self._h, int(token), ctypes.byref(self._logits))
        return list(self._logits)

    def prefill(self, tokens) -> list:
        toks = list(tokens)
        buf = (ctypes.c_int * len(toks))(*toks)
        self._lib.sn_prefill(self._h, buf, len(toks), ctypes.byref(self._logits))
        return list(self._logits)

    def dbg_layer(self, token: int, layer: int, n: int) -> list:
        buf = (ctypes.c_float * n)()
        self._lib.sn_dbg_layer(self._h, int(token), int(layer), ctypes.byref(buf))
        return list(buf)

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                self._lib.sn_free(self._h)
        except Exception:
            pass
