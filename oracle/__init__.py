"""CPU oracle for the SunnyNet token loop -- TEST INFRASTRUCTURE ONLY.

Two checkers live here:

* ``liboracle.so`` (``oracle/sn_oracle.c``): this project's plain-C restatement of
  the reference runtime's arithmetic, bit-identical to it by construction.
* ``oracle/_ref/libsnref_*.so``: the reference runtime itself, compiled from its
  own unmodified sources by ``oracle/Makefile`` when the reference tree is
  present. It is used to pin the restatement and as the timed CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package; the product (``sunnynet_b200``) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_ABI_SO = HERE / "_ref" / "libsnref_abi.so"
REF_MODEL_SO = HERE / "_ref" / "libsnref_model.so"
REF_KERNELS_SO = HERE / "_ref" / "libsnref_kernels.so"

_F = ctypes.POINTER(ctypes.c_float)
_V, _I, _P = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p


def build(quiet: bool = True, ref_root=None) -> None:
    """Compile the restatement, and oracle/_ref from the reference's own runtime
    sources when `ref_root` (the reference checkout) is given and present."""
    cmd = ["make", "-C", str(HERE), "all"]
    if ref_root is not None and (Path(ref_root) / "sunnynet" / "runtime").is_dir():
        cmd.append(f"REF={Path(ref_root) / 'sunnynet' / 'runtime'}")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + (r.stderr or r.stdout)[-2000:])
    if not quiet:
        print(r.stdout)


def _stale(so: Path, srcs) -> bool:
    if not so.exists():
        return True
    t = so.stat().st_mtime
    return any(s.exists() and s.stat().st_mtime > t for s in srcs)


_lib = None
_ref_abi = None
_ref_model = None
_ref_kernels = None


def lib():
    """Load liboracle.so, building it first if needed."""
    global _lib
    if _lib is not None:
        return _lib
    if _stale(ORACLE_SO, [HERE / "sn_oracle.c", HERE / "sn_oracle.h"]):
        build()
    L = ctypes.CDLL(str(ORACLE_SO))
    L.or_recur_scan.argtypes = [_V, _V, _V, _V, _V, _I, _I, _I, _I]
    L.or_recur_step.argtypes = [_V, _V, _V, _I, _I, _I]
    L.or_recur_bwd.argtypes = [_V, _V, _V, _V, _V, _V, _V, _V, _I, _I, _I, _I]
    L.or_quant_i8.argtypes = [_V, _V, _V, _I, _I, _I]
    L.or_dequant_i8.argtypes = [_V, _V, _V, _I, _I, _I]
    L.or_quant_i4.argtypes = [_V, _V, _V, _I, _I, _I, _I]
    L.or_dequant_i4.argtypes = [_V, _V, _V, _I, _I, _I, _I]
    L.or_gemv_i4.argtypes = [_V, _V, _V, _V, _I, _I, _I, _I]
    L.or_gemv_i4.restype = _I
    L.or_gemv_f32.argtypes = [_V, _V, _V, _I, _I]
    L.or_sn_load.argtypes = [_P, _I]
    L.or_sn_load.restype = _V
    L.or_sn_free.argtypes = [_V]
    L.or_sn_reset.argtypes = [_V]
    L.or_sn_vocab.argtypes = [_V]
    L.or_sn_vocab.restype = _I
    L.or_sn_step.argtypes = [_V, _V, _V]
    L.or_sn_dbg_layer.argtypes = [_V, _I, _I, _V]
    L.or_sn_get_state.argtypes = [_V, _I, _V, _V]
    L.or_sn_set_state.argtypes = [_V, _I, _V, _V]
    L.or_rk_load.argtypes = [_P, _I]
    L.or_rk_load.restype = _V
    L.or_rk_free.argtypes = [_V]
    L.or_rk_reset.argtypes = [_V]
    L.or_rk_vocab.argtypes = [_V]
    L.or_rk_vocab.restype = _I
    L.or_rk_step.argtypes = [_V, _V, _V]
    L.or_rk_dbg.argtypes = [_V, _I, _I, _V]
    L.or_rk_get_state.argtypes = [_V, _I, _V, _V]
    L.or_core_fwd.argtypes = [_V] * 6 + [_I] * 3
    L.or_core_bwd.argtypes = [_V] * 11 + [_I] * 3
    L.or_step_core.argtypes = [_V] * 5 + [_I] * 2
    L.or_dw_step.argtypes = [_V] * 4 + [_I] * 3
    L.or_scan_f32.argtypes = [_V] * 5 + [_I] * 3
    L.or_rk_set_state.argtypes = [_V, _I, _V, _V]
    L.or_rk_step_forced.argtypes = [_V, _V, _V, _V, _V]
    _lib = L
    return L


def ref_available() -> bool:
    """True when oracle/_ref holds the reference runtime built from its sources."""
    return REF_ABI_SO.exists() and REF_MODEL_SO.exists()


def ref_abi():
    """The reference's sn_abi + recur + rwkv7 + quant library (oracle/_ref)."""
    global _ref_abi
    if _ref_abi is None:
        if not REF_ABI_SO.exists():
            raise FileNotFoundError(REF_ABI_SO)
        L = ctypes.CDLL(str(REF_ABI_SO))
        L.sn_recur_scan.argtypes = [_V, _V, _V, _V, _V, _I, _I, _I, _I]
        L.sn_recur_step.argtypes = [_V, _V, _V, _I, _I, _I]
        L.sn_recur_bwd.argtypes = [_V, _V, _V, _V, _V, _V, _V, _V, _I, _I, _I, _I]
        L.sn_quant_i8.argtypes = [_V, _V, _V, _I, _I, _I]
        L.sn_dequant_i8.argtypes = [_V, _V, _V, _I, _I, _I]
        L.sn_quant_i4.argtypes = [_V, _V, _V, _I, _I, _I]
        L.sn_dequant_i4.argtypes = [_V, _V, _V, _I, _I, _I]
        L.sn_gemv_i4.argtypes = [_V, _V, _V, _V, _I, _I, _I]
        L.sn_gemv_f32.argtypes = [_V, _V, _V, _I, _I]
        L.sn_set_threads.argtypes = [_I]
        L.sn_threads.restype = _I
        L.sn_rk_load.argtypes = [_P]
        L.sn_rk_load.restype = _V
        L.sn_rk_free.argtypes = [_V]
        L.sn_rk_reset.argtypes = [_V]
        L.sn_rk_step.argtypes = [_V, _I, _V]
        L.sn_rk_prefill.argtypes = [_V, _V, _I, _V]
        L.sn_rk_dbg.argtypes = [_V, _I, _I, _V]
        L.sn_rk_vocab.argtypes = [_V]
        L.sn_rk_vocab.restype = _I
        _ref_abi = L
    return _ref_abi


def ref_model():
    """The reference's sunnynet.c whole-model library (oracle/_ref)."""
    global _ref_model
    if _ref_model is None:
        if not REF_MODEL_SO.exists():
            raise FileNotFoundError(REF_MODEL_SO)
        L = ctypes.CDLL(str(REF_MODEL_SO))
        L.sn_load.restype = _V
        L.sn_load.argtypes = [_P, _I, _I, _I, _I, _I, _I, _I, _I]
        L.sn_load_h.restype = _V
        L.sn_load_h.argtypes = [_P, _I, _I, _I, _I, _I, _I, _I, _I]
        L.sn_free.argtypes = [_V]
        L.sn_reset.argtypes = [_V]
        L.sn_step.argtypes = [_V, _I, _V]
        L.sn_prefill.argtypes = [_V, _V, _I, _V]
        L.sn_dbg_layer.argtypes = [_V, _I, _I, _V]
        L.sn_vocab.argtypes = [_V]
        L.sn_vocab.restype = _I
        L.sn_set_threads.argtypes = [_I]
        L.sn_get_threads.restype = _I
        L.sn_recommended_threads.restype = _I
        _ref_model = L
    return _ref_model


def ref_kernels():
    """The reference's kernels module (scan_avx2.c, core_avx2.c, step_avx2.c)
    built with its own flags into oracle/_ref, bound as kernels/__init__.py
    binds it."""
    global _ref_kernels
    if _ref_kernels is None:
        if not REF_KERNELS_SO.exists():
            raise FileNotFoundError(REF_KERNELS_SO)
        L = ctypes.CDLL(str(REF_KERNELS_SO))
        L.scan_f32.argtypes = [_V] * 5 + [_I] * 3
        L.scan_bwd_f32.argtypes = [_V] * 8 + [_I] * 3
        L.core_fwd_f32.argtypes = [_V] * 6 + [_I] * 3
        L.core_bwd_f32.argtypes = [_V] * 11 + [_I] * 3
        L.dw_step_f32.argtypes = [_V] * 4 + [_I] * 3
        L.step_core_f32.argtypes = [_V] * 5 + [_I] * 2
        L.sn_set_threads.argtypes = [_I]
        _ref_kernels = L
    return _ref_kernels


def ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


# ------------------------------------------------------------ array helpers
def recur_scan(a, b, s0, gated):
    B, T, N = a.shape
    out = np.empty_like(a)
    send = np.empty((B, N), np.float32)
    lib().or_recur_scan(ptr(a), ptr(b), ptr(s0), ptr(out), ptr(send), B, T, N, int(gated))
    return out, send


def recur_bwd(a, b, s0, out, dout, gated):
    """Reverse pass of the scan (reference recur.c:51-107) -> (da, db, ds0)."""
    B, T, N = a.shape
    da = np.empty_like(a)
    db = np.empty_like(a)
    ds0 = np.empty((B, N), np.float32)
    lib().or_recur_bwd(ptr(a), ptr(b), ptr(s0), ptr(out), ptr(dout), ptr(da), ptr(db), ptr(ds0),
                       B, T, N, int(gated))
    return da, db, ds0


def core_fwd(q, delta, s0):
    """core_avx2.c core_fwd_f32: q (B,T,2D), delta (D), s0 (B,D) -> states, u, p."""
    B, T, D2 = q.shape
    D = D2 // 2
    st, u, p = (np.zeros((B, T, D), np.float32) for _ in range(3))
    lib().or_core_fwd(ptr(q), ptr(delta), ptr(s0), ptr(st), ptr(u), ptr(p), B, T, D)
    return st, u, p


def core_bwd(q, delta, s0, states, u, p, dstate, du):
    """core_avx2.c core_bwd_f32 -> (dq, ddelta, ds0)."""
    B, T, D2 = q.shape
    D = D2 // 2
    dq = np.zeros_like(q)
    dd = np.zeros(D, np.float32)
    ds0 = np.zeros((B, D), np.float32)
    lib().or_core_bwd(ptr(q), ptr(delta), ptr(s0), ptr(states), ptr(u), ptr(p), ptr(dstate),
                      ptr(du), ptr(dq), ptr(dd), ptr(ds0), B, T, D)
    return dq, dd, ds0


def step_core(q, delta, s):
    """step_avx2.c step_core_f32: q (B,2D), s (B,D) -> (u, s_new)."""
    B, D2 = q.shape
    D = D2 // 2
    sn = np.zeros((B, D), np.float32)
    u = np.zeros((B, D), np.float32)
    lib().or_step_core(ptr(q), ptr(delta), ptr(s), ptr(sn), ptr(u), B, D)
    return u, sn


def scan_f32(p, nu, s0):
    """scan_avx2.c scan_f32: s = p*s + (1-p)*nu, lane rule on every channel."""
    B, T, N = p.shape
    out = np.empty_like(p)
    send = np.empty((B, N), np.float32)
    lib().or_scan_f32(ptr(p), ptr(nu), ptr(s0), ptr(out), ptr(send), B, T, N)
    return out, send


def dw_step(x, hist, w):
    """step_avx2.c dw_step_f32: x (B,D), hist (B,K-1,D), w (K,D) -> acc (B,D)."""
    B, D = x.shape
    acc = np.empty((B, D), np.float32)
    lib().or_dw_step(ptr(x), ptr(hist), ptr(w), ptr(acc), B, D, w.shape[0])
    return acc


def recur_step(a, b, s, gated):
    B, N = a.shape
    s = s.copy()
    lib().or_recur_step(ptr(a), ptr(b), ptr(s), B, N, int(gated))
    return s


def quant_i8(x, block):
    B, N = x.shape
    nb = (N + block - 1) // block if block > 0 else 1
    q = np.empty((B, N), np.int8)
    sc = np.empty((B, nb), np.float32)
    lib().or_quant_i8(ptr(x), ptr(q), ptr(sc), B, N, block)
    return q, sc


def dequant_i8(q, sc, block):
    B, N = q.shape
    x = np.empty((B, N), np.float32)
    lib().or_dequant_i8(ptr(q), ptr(sc), ptr(x), B, N, block)
    return x


def quant_i4(x, block, fp16=False):
    rows, N = x.shape
    q = np.empty((rows, N // 2), np.uint8)
    sc = np.empty((rows, N // block), np.float16 if fp16 else np.float32)
    lib().or_quant_i4(ptr(x), ptr(q), ptr(sc), rows, N, block, int(fp16))
    return q, sc


def dequant_i4(q, sc, N, block):
    rows = q.shape[0]
    x = np.empty((rows, N), np.float32)
    lib().or_dequant_i4(ptr(q), ptr(sc), ptr(x), rows, N, block, int(sc.dtype == np.float16))
    return x


def gemv_i4(x, q, sc, block):
    out = q.shape[0]
    y = np.empty(out, np.float32)
    rc = lib().or_gemv_i4(ptr(y), ptr(x), ptr(q), ptr(sc), x.shape[0], out, block,
                          int(sc.dtype == np.float16))
    if rc != 0:
        raise ValueError("unsupported W4A8 shape")
    return y


class Sunny:
    """Oracle SunnyNet handle over `nseq` independent sequences."""

    def __init__(self, path, nseq=1):
        self.L = lib()
        self.h = self.L.or_sn_load(str(path).encode(), nseq)
        if not self.h:
            raise RuntimeError(f"oracle could not load {path}")
        self.nseq = nseq
        self.vocab = self.L.or_sn_vocab(self.h)

    def step(self, tokens, want_logits=True):
        t = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(self.nseq))
        lg = np.empty((self.nseq, self.vocab), np.float32) if want_logits else None
        self.L.or_sn_step(self.h, ptr(t), ptr(lg) if want_logits else None)
        return lg

    def reset(self):
        self.L.or_sn_reset(self.h)

    def dbg_layer(self, token, layer, n):
        out = np.empty(n, np.float32)
        self.L.or_sn_dbg_layer(self.h, int(token), int(layer), ptr(out))
        return out

    def get_state(self, seq, L, D, KH):
        s = np.empty((L, D), np.float32)
        h = np.empty((L, KH, D), np.float32)
        self.L.or_sn_get_state(self.h, seq, ptr(s), ptr(h))
        return s, h

    def set_state(self, seq, s, h):
        s = np.ascontiguousarray(s, np.float32)
        h = np.ascontiguousarray(h, np.float32)
        self.L.or_sn_set_state(self.h, seq, ptr(s), ptr(h))

    def __del__(self):
        try:
            if self.h:
                self.L.or_sn_free(self.h)
        except Exception:
            pass


class Rwkv:
    """Oracle RWKV-7 handle over `nseq` independent sequences."""

    def __init__(self, path, nseq=1):
        self.L = lib()
        self.h = self.L.or_rk_load(str(path).encode(), nseq)
        if not self.h:
            raise RuntimeError(f"oracle could not load {path}")
        self.nseq = nseq
        self.vocab = self.L.or_rk_vocab(self.h)

    def step(self, tokens, want_logits=True):
        t = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(self.nseq))
        lg = np.empty((self.nseq, self.vocab), np.float32) if want_logits else None
        self.L.or_rk_step(self.h, ptr(t), ptr(lg) if want_logits else None)
        return lg

    def reset(self):
        self.L.or_rk_reset(self.h)

    def dbg(self, token, layer, D):
        out = np.empty(9 * D, np.float32)
        self.L.or_rk_dbg(self.h, int(token), int(layer), ptr(out))
        return out

    def set_state(self, seq, S, shift):
        S = np.ascontiguousarray(S, np.float32)
        shift = np.ascontiguousarray(shift, np.float32)
        self.L.or_rk_set_state(self.h, seq, ptr(S), ptr(shift))

    def step_forced(self, tokens, xs_in):
        """Each layer of each sequence run from xs_in (nseq, L+1, D), the input
        another implementation gave it -> (xs_out (nseq, L+1, D), logits)."""
        t = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(self.nseq))
        xs_in = np.ascontiguousarray(xs_in, np.float32)
        xs_out = np.empty_like(xs_in)
        lg = np.empty((self.nseq, self.vocab), np.float32)
        self.L.or_rk_step_forced(self.h, ptr(t), ptr(xs_in), ptr(xs_out), ptr(lg))
        return xs_out, lg

    def get_state(self, seq, L, NH, HS, D):
        S = np.empty((L, NH, HS, HS), np.float32)
        sh = np.empty((L, 2, D), np.float32)
        self.L.or_rk_get_state(self.h, seq, ptr(S), ptr(sh))
        return S, sh

    def __del__(self):
        try:
            if self.h:
                self.L.or_rk_free(self.h)
        except Exception:
            pass


def set_threads(n: int) -> None:
    os.environ["OMP_NUM_THREADS"] = str(n)
