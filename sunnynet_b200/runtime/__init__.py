"""SunnyNet runtime on a B200: the recurrence kernels behind the C ABI.

Mirrors the reference's ``sunnynet/runtime/__init__.py`` (FMA/GATED forms,
``scan``/``step``/``quant_i8``/``dequant_i8``, ``load_runtime``) so callers can
switch imports. Arguments are torch tensors (CPU or CUDA) or numpy arrays;
results come back in the same kind and on the same device::

    s_t = a_t * s_{t-1} + b_t          (FMA)
    s_t = a_t * s_{t-1} + (1-a_t)*u_t  (GATED)

Results are bit-identical to the reference AVX2 runtime.
"""
from __future__ import annotations

import numpy as np

from .. import _lib
from .._lib import check, ptr

__all__ = ["runtime_available", "load_runtime", "FMA", "GATED", "scan", "scan_bwd", "step",
           "quant_i8",
           "dequant_i8", "quant_i4", "dequant_i4", "gemv_i4", "gemm_i4", "gemv_f32",
           "bind_stream", "set_scan_mode"]

FMA = 0
GATED = 1


def runtime_available() -> bool:
    return _lib.LIB_PATH.exists()


def load_runtime(force_rebuild: bool = False):
    if force_rebuild or not _lib.LIB_PATH.exists():
        from .. import build
        build.build(force=force_rebuild)
    return _lib.load()


def _is_torch(x) -> bool:
    return hasattr(x, "data_ptr")


def bind_stream(*xs) -> None:
    """Run the library on torch's current stream when CUDA tensors are involved,
    so its kernels are ordered after the work that produced them."""
    for x in xs:
        if _is_torch(x) and x.is_cuda:
            import torch
            check(_lib.load().sn_abi_cuda_set_stream(
                torch.cuda.current_stream(x.device).cuda_stream), "set_stream")
            return


def _empty(like, shape, dtype):
    if _is_torch(like):
        import torch
        tdt = {np.float32: torch.float32, np.int8: torch.int8, np.uint8: torch.uint8,
               np.float16: torch.float16}[dtype]
        return torch.empty(shape, dtype=tdt, device=like.device)
    return np.empty(shape, dtype)


def set_scan_mode(mode: int) -> int:
    """Select the scan algorithm of ``scan``; returns the previous mode.

    0 (default): sequential in T per channel, bit-identical to the reference.
    1: chunked in T (per-chunk affine maps composed into the carry entering
    each chunk), many times more parallel; outputs within a few ulp of the
    state per chunk boundary of mode 0 instead of bit-identical.
    """
    return int(load_runtime().sn_abi_cuda_scan_mode(int(mode)))


def scan(a, b, s0, gated=False):
    """a, b: (B,T,N); s0: (B,N) -> (out (B,T,N), send (B,N))."""
    lib = load_runtime()
    B, T, N = a.shape
    out = _empty(a, (B, T, N), np.float32)
    send = _empty(a, (B, N), np.float32)
    bind_stream(a, b, s0)
    check(lib.sn_abi_recur_scan(ptr(a), ptr(b), ptr(s0), ptr(out), ptr(send), B, T, N,
                                GATED if gated else FMA), "recur_scan")
    return out, send


def scan_bwd(a, b, s0, out, dout, gated=False):
    """Reverse pass over ``scan``'s outputs -> (da, db, ds0) (reference
    runtime/__init__.py ``scan_bwd``, recur.c:51-107); gated: b holds u and
    (da, db) are the gradients w.r.t. a and u. Bit-identical to the reference."""
    lib = load_runtime()
    B, T, N = a.shape
    da = _empty(a, (B, T, N), np.float32)
    db = _empty(a, (B, T, N), np.float32)
    ds0 = _empty(a, (B, N), np.float32)
    bind_stream(a, b, s0, out, dout)
    check(lib.sn_abi_recur_bwd(ptr(a), ptr(b), ptr(s0), ptr(out), ptr(dout), ptr(da), ptr(db),
                               ptr(ds0), B, T, N, GATED if gated else FMA), "recur_bwd")
    return da, db, ds0


def step(a, b, s, gated=False):
    """a, b, s: (B,N); s updated in place and returned."""
    lib = load_runtime()
    B, N = a.shape
    bind_stream(a, b, s)
    check(lib.sn_abi_recur_step(ptr(a), ptr(b), ptr(s), B, N, GATED if gated else FMA),
          "recur_step")
    return s


def quant_i8(x, block: int = 0):
    """x (B,N) fp32 -> (q int8 (B,N), scale (B,nb) fp32)."""
    lib = load_runtime()
    B, N = x.shape
    nb = (N + block - 1) // block if block > 0 else 1
    q = _empty(x, (B, N), np.int8)
    sc = _empty(x, (B, nb), np.float32)
    bind_stream(x)
    check(lib.sn_abi_quant_i8(ptr(x), ptr(q), ptr(sc), B, N, block), "quant_i8")
    return q, sc


def dequant_i8(q, scale, block: int = 0):
    lib = load_runtime()
    B, N = q.shape
    x = _empty(q, (B, N), np.float32)
    bind_stream(q, scale)
    check(lib.sn_abi_dequant_i8(ptr(q), ptr(scale), ptr(x), B, N, block), "dequant_i8")
    return x


def _fp16(sc) -> int:
    dt = getattr(sc, "dtype", None)
    return int(str(dt) in ("float16", "torch.float16"))


def quant_i4(x, block: int = 64, fp16_scale: bool = False):
    """x (rows,N) fp32 -> (codes uint8 (rows,N/2), scale (rows,N/block))."""
    lib = load_runtime()
    rows, N = x.shape
    q = _empty(x, (rows, N // 2), np.uint8)
    sc = _empty(x, (rows, N // block), np.float16 if fp16_scale else np.float32)
    bind_stream(x)
    check(lib.sn_abi_quant_i4(ptr(x), ptr(q), ptr(sc), rows, N, block, int(fp16_scale)),
          "quant_i4")
    return q, sc


def dequant_i4(q, scale, N: int, block: int = 64):
    lib = load_runtime()
    rows = q.shape[0]
    x = _empty(q, (rows, N), np.float32)
    bind_stream(q, scale)
    check(lib.sn_abi_dequant_i4(ptr(q), ptr(scale), ptr(x), rows, N, block, _fp16(scale)),
          "dequant_i4")
    return x


def gemv_i4(x, q, scale, block: int = 64):
    """y = W x with W given as INT4 (codes (out,in/2), scales); W4A8 semantics."""
    lib = load_runtime()
    n = x.shape[0]
    out = q.shape[0]
    y = _empty(x, (out,), np.float32)
    bind_stream(x, q, scale)
    check(lib.sn_abi_gemv_i4(ptr(y), ptr(x), ptr(q), ptr(scale), n, out, block, _fp16(scale)),
          "gemv_i4")
    return y


def gemm_i4(X, q, scale, block: int = 64):
    """Y (B,out) = each row of X (B,in) through the W4A8 GEMV."""
    lib = load_runtime()
    B, n = X.shape
    out = q.shape[0]
    Y = _empty(X, (B, out), np.float32)
    bind_stream(X, q, scale)
    check(lib.sn_abi_gemm_i4(ptr(Y), ptr(X), ptr(q), ptr(scale), B, n, out, block, _fp16(scale)),
          "gemm_i4")
    return Y


def gemv_f32(x, W):
    lib = load_runtime()
    out, n = W.shape
    y = _empty(x, (out,), np.float32)
    bind_stream(x, W)
    lib.sn_gemv_f32(ptr(y), ptr(x), ptr(W), n, out)
    return y
