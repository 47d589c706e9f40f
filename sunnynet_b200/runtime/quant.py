"""INT4 primitives (numpy in, numpy out), mirroring the reference's
``sunnynet/runtime/quant.py``: quant_i4 / dequant_i4 / gemv_i4 / gemv_f32."""
from __future__ import annotations

import numpy as np

from . import dequant_i4 as _dequant_i4
from . import gemv_f32 as _gemv_f32
from . import gemv_i4 as _gemv_i4
from . import load_runtime
from . import quant_i4 as _quant_i4

__all__ = ["quant_available", "load_quant", "I4_BLOCK", "quant_i4", "dequant_i4", "gemv_i4",
           "gemv_f32"]

I4_BLOCK = 64


def quant_available() -> bool:
    from .. import _lib
    return _lib.LIB_PATH.exists()


def load_quant(force_rebuild: bool = False):
    return load_runtime(force_rebuild)


def quant_i4(x, block: int = I4_BLOCK):
    return _quant_i4(np.ascontiguousarray(x, np.float32), block)


def dequant_i4(q, scale, N: int, block: int = I4_BLOCK):
    return _dequant_i4(np.ascontiguousarray(q, np.uint8), np.ascontiguousarray(scale), N, block)


def gemv_i4(x, q, scale, block: int = I4_BLOCK):
    return _gemv_i4(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(q, np.uint8),
                    np.ascontiguousarray(scale), block)


def gemv_f32(x, W):
    return _gemv_f32(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(W, np.float32))
