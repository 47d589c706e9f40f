"""The reference's hand-written kernels module on a B200: the loader and the
torch autograd operators of ``sunnynet/kernels`` (``__init__.py``,
``core_auto.py``, ``scan_auto.py``), backed by libsunnynet_cuda.so.

Same names and argument meaning, so training code switches by import:
``load_kernel`` / ``load_scan_kernel`` return the library with the argtypes
set; ``CoreCUDA`` (the reference's ``CoreAVX2``) takes q (B,T,2D) = [u_raw |
gate], delta (D,), s0 (B,D) and returns (u, states); ``ScanCUDA`` (the
reference's ``ScanAVX2``) takes u, p (B,T,N), s0 (B,N) and returns the states;
``step_core`` and ``dw_step`` are the decode-time single steps. Tensors may be
on the GPU (then the kernels read them in place, on torch's current stream)
or on the host (staged through device memory). There is no CPU fallback.
"""
from __future__ import annotations

from . import _lib
from ._lib import ptr
from .runtime import bind_stream, load_runtime

__all__ = ["load_kernel", "load_scan_kernel", "kernel_available", "set_kernel_threads",
           "CoreCUDA", "core_forward", "step_core", "dw_step", "ScanCUDA", "scan_auto"]


def load_kernel(force_rebuild: bool = False):
    """The library, with the argtypes of the kernels module set."""
    return load_runtime(force_rebuild)


def load_scan_kernel(force_rebuild: bool = False):
    return load_kernel(force_rebuild)


def kernel_available() -> bool:
    return _lib.LIB_PATH.exists()


def set_kernel_threads(n: int) -> None:
    """Kept for the reference's interface; the GPU ignores host thread counts."""
    load_kernel().sn_set_threads(int(n))


def _call(name: str, *args) -> None:
    """Call a void entry point; its failure is the message it leaves."""
    lib = load_kernel()
    lib.sn_abi_clear_error()
    getattr(lib, name)(*args)
    msg = _lib.last_error()
    if msg:
        raise _lib.SnError(-1, f"{name}: {msg}")


def _f32(t):
    return t.contiguous().float()


class CoreCUDA:
    """Fused competition gate + decay gate + scan as an autograd operator:
    (q, delta, s0) -> (u, states) (reference core_auto.CoreAVX2)."""

    @staticmethod
    def apply(q, delta, s0):
        return _core_fn().apply(q, delta, s0)


_CORE = None


def _core_fn():
    global _CORE
    if _CORE is not None:
        return _CORE
    import torch

    class _Core(torch.autograd.Function):
        @staticmethod
        def forward(ctx, q, delta, s0):
            B, T, D2 = q.shape
            D = D2 // 2
            q_c, delta_c, s0_c = _f32(q), _f32(delta), _f32(s0)
            states = torch.empty(B, T, D, dtype=torch.float32, device=q.device)
            u = torch.empty_like(states)
            p = torch.empty_like(states)
            bind_stream(q_c)
            _call("core_fwd_f32", ptr(q_c), ptr(delta_c), ptr(s0_c), ptr(states), ptr(u),
                  ptr(p), B, T, D)
            ctx.save_for_backward(q_c, delta_c, s0_c, states, u, p)
            return u, states

        @staticmethod
        def backward(ctx, du, dstate):
            q_c, delta_c, s0_c, states, u, p = ctx.saved_tensors
            B, T, D2 = q_c.shape
            D = D2 // 2
            du = torch.zeros_like(u) if du is None else _f32(du)
            dstate = torch.zeros_like(states) if dstate is None else _f32(dstate)
            dq = torch.empty_like(q_c)
            ddelta = torch.zeros(D, dtype=torch.float32, device=q_c.device)
            ds0 = torch.empty_like(s0_c)
            bind_stream(q_c)
            _call("core_bwd_f32", ptr(q_c), ptr(delta_c), ptr(s0_c), ptr(states), ptr(u),
                  ptr(p), ptr(dstate), ptr(du), ptr(dq), ptr(ddelta), ptr(ds0), B, T, D)
            return dq, ddelta, ds0

    _CORE = _Core
    return _CORE


def core_forward(q, delta, s0):
    """(u, states) of the fused core (reference core_auto.core_forward)."""
    return CoreCUDA.apply(q, delta, s0)


def step_core(q, delta, s):
    """One decode step: q (B,2D), delta (D,), s (B,D) -> (u, s_new)
    (reference core_auto.step_core)."""
    import torch
    B, D2 = q.shape
    D = D2 // 2
    q, delta, s = _f32(q), _f32(delta), _f32(s)
    s_new = torch.empty_like(s)
    u = torch.empty(B, D, dtype=torch.float32, device=q.device)
    bind_stream(q)
    _call("step_core_f32", ptr(q), ptr(delta), ptr(s), ptr(s_new), ptr(u), B, D)
    return u, s_new


def dw_step(x, hist, w_t, taps: int):
    """Depthwise causal taps, one step: x (B,D), hist (B,taps-1,D), w (taps,D)
    -> acc (B,D) (reference core_auto.dw_step)."""
    import torch
    B, D = x.shape
    x, hist, w_t = _f32(x), _f32(hist), _f32(w_t)
    acc = torch.empty(B, D, dtype=torch.float32, device=x.device)
    bind_stream(x)
    _call("dw_step_f32", ptr(x), ptr(hist), ptr(w_t), ptr(acc), B, D, int(taps))
    return acc


_SCAN = None


def _scan_fn():
    global _SCAN
    if _SCAN is not None:
        return _SCAN
    import torch

    class _Scan(torch.autograd.Function):
        @staticmethod
        def forward(ctx, u, p, s0):
            B, T, N = u.shape
            u_c, p_c, s0_c = _f32(u), _f32(p), _f32(s0)
            out = torch.empty_like(u_c)
            send = torch.empty_like(s0_c)
            bind_stream(u_c)
            _call("scan_f32", ptr(p_c), ptr(u_c), ptr(s0_c), ptr(out), ptr(send), B, T, N)
            ctx.save_for_backward(u_c, p_c, s0_c, out)
            return out

        @staticmethod
        def backward(ctx, dout):
            u_c, p_c, s0_c, out = ctx.saved_tensors
            B, T, N = u_c.shape
            dout_c = _f32(dout)
            dp = torch.empty_like(p_c)
            du = torch.empty_like(u_c)
            ds0 = torch.empty_like(s0_c)
            bind_stream(u_c)
            _call("scan_bwd_f32", ptr(p_c), ptr(u_c), ptr(s0_c), ptr(out), ptr(dout_c),
                  ptr(dp), ptr(du), ptr(ds0), B, T, N)
            return du, dp, ds0

    _SCAN = _Scan
    return _SCAN


class ScanCUDA:
    """s_t = p_t*s_{t-1} + (1-p_t)*u_t forward and backward as an autograd
    operator: (u, p, s0) -> states (reference scan_auto.ScanAVX2)."""

    @staticmethod
    def apply(u, p, s0):
        return _scan_fn().apply(u, p, s0)


def scan_auto(u, p, s0, chunk: int = 64, p_min_hint=None):
    """(states, last state) of the gated scan (reference scan_auto.scan_auto;
    chunk and p_min_hint only steer the reference's torch fallback, which this
    module does not have)."""
    states = ScanCUDA.apply(u, p, s0)
    return states, states[:, -1]
