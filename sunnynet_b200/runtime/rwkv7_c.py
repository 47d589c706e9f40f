"""B=1 RWKV-7 handle over the reference's internal ABI (rwkv7.h), on a B200.

Same class as the reference's ``sunnynet/runtime/rwkv7_c.py`` (``SnRWKV7`` with
reset/step/step_raw/logits/prefill/dbg) so ``--gguf-backend`` can pick it.
"""
from __future__ import annotations

import ctypes

from .. import _lib
from . import load_runtime

__all__ = ["SnRWKV7", "rwkv7_available"]


def rwkv7_available() -> bool:
    return _lib.LIB_PATH.exists()


class SnRWKV7:
    def __init__(self, path, vocab: int):
        self._lib = load_runtime()
        self._logits = (ctypes.c_float * vocab)()
        self._h = self._lib.sn_rk_load(str(path).encode())
        if not self._h:
            raise RuntimeError(f"sn_rk_load failed: {path} ({_lib.last_error()})")
        if not self._lib.sn_rk_ready(self._h):
            raise RuntimeError("sn_rk_load returned a handle that is not ready")
        self.vocab = vocab

    def reset(self):
        self._lib.sn_rk_reset(self._h)

    def step(self, token: int) -> list:
        self._lib.sn_rk_step(self._h, int(token), ctypes.byref(self._logits))
        return list(self._logits)

    def step_raw(self, token: int) -> None:
        self._lib.sn_rk_step(self._h, int(token), ctypes.byref(self._logits))

    def logits(self) -> list:
        return list(self._logits)

    def prefill(self, tokens) -> list:
        toks = list(tokens)
        buf = (ctypes.c_int * len(toks))(*toks)
        self._lib.sn_rk_prefill(self._h, buf, len(toks), ctypes.byref(self._logits))
        return list(self._logits)

    def dbg(self, token: int, layer: int, dim: int) -> list:
        buf = (ctypes.c_float * (9 * dim))()
        self._lib.sn_rk_dbg(self._h, int(token), int(layer), ctypes.byref(buf))
        return list(buf)

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                self._lib.sn_rk_free(self._h)
        except Exception:
            pass
