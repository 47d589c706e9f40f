"""ctypes binding of libsunnynet_cuda.so (the C ABI in include/*.h).

There is no fallback: if the library is missing or the device is not an
sm_100 part, calls raise. Array arguments may be numpy arrays (host memory)
or torch tensors (host or CUDA); the library tells host from device memory.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsunnynet_cuda.so"

V, I32, U32, P = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_char_p
CI = ctypes.c_int

# name -> (restype, argtypes); every symbol declared in include/*.h
SIGNATURES = {
    # sn_abi.h, ABI 1.0
    "sn_abi_version": (I32, []),
    "sn_abi_caps": (U32, []),
    "sn_abi_check": (I32, [I32]),
    "sn_abi_version_string": (I32, [P, I32]),
    "sn_abi_backend_string": (I32, [P, I32]),
    "sn_abi_set_threads": (I32, [I32]),
    "sn_abi_get_threads": (I32, []),
    "sn_abi_recur_step": (I32, [V, V, V, I32, I32, I32]),
    "sn_abi_recur_scan": (I32, [V, V, V, V, V, I32, I32, I32, I32]),
    "sn_abi_recur_scan_noalloc": (I32, [V, V, V, V, V, I32, I32, I32, I32, V]),
    "sn_abi_recur_bwd": (I32, [V, V, V, V, V, V, V, V, I32, I32, I32, I32]),
    "sn_abi_quant_i8": (I32, [V, V, V, I32, I32, I32]),
    "sn_abi_dequant_i8": (I32, [V, V, V, I32, I32, I32]),
    "sn_abi_rwkv7_load": (V, [P]),
    "sn_abi_rwkv7_step": (I32, [V, I32, V]),
    "sn_abi_rwkv7_prefill": (I32, [V, V, I32, V]),
    "sn_abi_rwkv7_reset": (I32, [V]),
    "sn_abi_rwkv7_free": (None, [V]),
    "sn_abi_rwkv7_vocab": (I32, [V]),
    # sn_abi.h, ABI 1.1
    "sn_abi_cuda_set_stream": (I32, [V]),
    "sn_abi_cuda_set_async": (I32, [I32]),
    "sn_abi_cuda_synchronize": (I32, []),
    "sn_abi_last_error": (I32, [P, I32]),
    "sn_abi_clear_error": (None, []),
    "sn_abi_cuda_scan_mode": (I32, [I32]),
    "sn_abi_cuda_int8_mainloop": (I32, [I32]),
    "sn_abi_cuda_profile": (I32, [I32]),
    "sn_abi_cuda_profile_report": (I32, [P, I32]),
    "sn_abi_cuda_wait_selftest": (I32, [I32, ctypes.c_int64]),
    "sn_abi_quant_i4": (I32, [V, V, V, I32, I32, I32, I32]),
    "sn_abi_dequant_i4": (I32, [V, V, V, I32, I32, I32, I32]),
    "sn_abi_gemv_i4": (I32, [V, V, V, V, I32, I32, I32, I32]),
    "sn_abi_gemm_i4": (I32, [V, V, V, V, I32, I32, I32, I32, I32]),
    "sn_abi_sunny_load": (V, [P, I32]),
    "sn_abi_sunny_free": (None, [V]),
    "sn_abi_sunny_reset": (I32, [V]),
    "sn_abi_sunny_vocab": (I32, [V]),
    "sn_abi_sunny_dims": (I32, [V, V]),
    "sn_abi_sunny_step": (I32, [V, V, I32, V]),
    "sn_abi_sunny_step_argmax": (I32, [V, V, I32, V]),
    "sn_abi_sunny_prefill": (I32, [V, V, I32, I32, V]),
    "sn_abi_sunny_prefill_chunked": (I32, [V, V, I32, I32, I32, V]),
    "sn_abi_sunny_get_state": (I32, [V, I32, V, V]),
    "sn_abi_sunny_set_state": (I32, [V, I32, V, V]),
    "sn_abi_sunny_get_state_at": (I32, [V, I32, I32, V, V]),
    "sn_abi_sunny_set_state_at": (I32, [V, I32, I32, V, V]),
    "sn_abi_sunny_reset_at": (I32, [V, I32, I32]),
    "sn_abi_rwkv7_load_batch": (V, [P, I32]),
    "sn_abi_rwkv7_step_batch": (I32, [V, V, I32, V]),
    "sn_abi_rwkv7_step_argmax": (I32, [V, V, I32, V]),
    "sn_abi_rwkv7_step_trace": (I32, [V, V, I32, V, V]),
    "sn_abi_rwkv7_prefill_batch": (I32, [V, V, I32, I32, V]),
    "sn_abi_rwkv7_get_state": (I32, [V, I32, V, V]),
    "sn_abi_rwkv7_dims": (I32, [V, V]),
    # recur.h
    "sn_set_threads": (None, [CI]),
    "sn_threads": (CI, []),
    "sn_recur_scan": (None, [V, V, V, V, V, CI, CI, CI, CI]),
    "sn_recur_step": (None, [V, V, V, CI, CI, CI]),
    "sn_recur_bwd": (None, [V, V, V, V, V, V, V, V, CI, CI, CI, CI]),
    "sn_quant_i8": (None, [V, V, V, CI, CI, CI]),
    "sn_dequant_i8": (None, [V, V, V, CI, CI, CI]),
    # quant.h
    "sn_quant_i4": (None, [V, V, V, CI, CI, CI]),
    "sn_dequant_i4": (None, [V, V, V, CI, CI, CI]),
    "sn_gemv_i4": (None, [V, V, V, V, CI, CI, CI]),
    "sn_gemv_f32": (None, [V, V, V, CI, CI]),
    # sunnynet.h
    "sn_load": (V, [P, CI, CI, CI, CI, CI, CI, CI, CI]),
    "sn_load_h": (V, [P, CI, CI, CI, CI, CI, CI, CI, CI]),
    "sn_free": (None, [V]),
    "sn_reset": (None, [V]),
    "sn_step": (None, [V, CI, V]),
    "sn_prefill": (None, [V, V, CI, V]),
    "sn_vocab": (CI, [V]),
    "sn_ready": (CI, [V]),
    "sn_get_threads": (CI, []),
    "sn_recommended_threads": (CI, []),
    "sn_dbg_layer": (None, [V, CI, CI, V]),
    # sn_kernels.h (the reference's kernels module)
    "scan_f32": (None, [V, V, V, V, V, CI, CI, CI]),
    "scan_bwd_f32": (None, [V, V, V, V, V, V, V, V, CI, CI, CI]),
    "core_fwd_f32": (None, [V, V, V, V, V, V, CI, CI, CI]),
    "core_bwd_f32": (None, [V, V, V, V, V, V, V, V, V, V, V, CI, CI, CI]),
    "step_core_f32": (None, [V, V, V, V, V, CI, CI]),
    "dw_step_f32": (None, [V, V, V, V, CI, CI, CI]),
    # rwkv7.h
    "sn_rk_load": (V, [P]),
    "sn_rk_free": (None, [V]),
    "sn_rk_reset": (None, [V]),
    "sn_rk_step": (None, [V, CI, V]),
    "sn_rk_prefill": (None, [V, V, CI, V]),
    "sn_rk_dbg": (None, [V, CI, CI, V]),
    "sn_rk_vocab": (CI, [V]),
    "sn_rk_ready": (CI, [V]),
}

STATUS = {0: "OK", -1: "E_INVAL", -2: "E_NOMEM", -3: "E_IO", -4: "E_FORMAT",
          -5: "E_UNSUPPORTED", -6: "E_DEVICE"}

_lib = None


class SnError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


def load():
    """Load the library (raises if it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is not built; run `python -m sunnynet_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    MISSING.clear()
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name, None)
        if f is None:
            MISSING.append(name)
            continue
        f.restype = res
        f.argtypes = args
    _lib = lib
    return lib


MISSING: list = []  # declared symbols the loaded library does not export


def last_error() -> str:
    lib = load()
    n = lib.sn_abi_last_error(None, 0)
    buf = ctypes.create_string_buffer(max(n, 1))
    lib.sn_abi_last_error(buf, n)
    return buf.value.decode(errors="replace")


def profile_report() -> dict:
    """{family: (launches, total_ms)} recorded since sn_abi_cuda_profile(1)."""
    import json
    lib = load()
    n = lib.sn_abi_cuda_profile_report(None, 0)
    buf = ctypes.create_string_buffer(n)
    lib.sn_abi_cuda_profile_report(buf, n)
    return {k: tuple(v) for k, v in json.loads(buf.value.decode()).items()}


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        raise SnError(int(rc), f"{what}: {last_error()}")


def ptr(x):
    """Raw address of a numpy array or torch tensor (None passes through)."""
    if x is None:
        return None
    if hasattr(x, "data_ptr"):
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return ctypes.c_void_p(x.data_ptr())
    if not x.flags["C_CONTIGUOUS"]:
        raise ValueError("array must be C-contiguous")
    return ctypes.c_void_p(x.ctypes.data)
