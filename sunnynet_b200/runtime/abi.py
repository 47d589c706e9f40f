"""ctypes view of the stable C ABI (sn_abi.h), mirroring the reference's
``sunnynet/runtime/abi.py``: version/caps/check/strings, status messages and
the ``Rwkv7ABI`` handle. The library is libsunnynet_cuda.so (backend "cuda")."""
from __future__ import annotations

import ctypes

from .. import _lib
from . import load_runtime

__all__ = ["abi_available", "load_abi", "ABI_VERSION", "CAPS", "STATUS_OK", "Rwkv7ABI"]

ABI_MAJOR, ABI_MINOR, ABI_PATCH = 1, 1, 0
ABI_VERSION = (ABI_MAJOR << 16) | (ABI_MINOR << 8) | ABI_PATCH

CAP_RECUR_SCAN = 1 << 0
CAP_RECUR_STEP = 1 << 1
CAP_QUANT_I8 = 1 << 2
CAP_RWKV7 = 1 << 3
CAP_THREADS = 1 << 4
CAP_CUDA = 1 << 5
CAP_QUANT_I4 = 1 << 6
CAP_SUNNY = 1 << 7
CAP_BATCH = 1 << 8
CAPS = ("recur_scan", "recur_step", "quant_i8", "rwkv7", "threads", "cuda", "quant_i4", "sunny",
        "batch")

STATUS_OK = 0
_STATUS_MSG = {
    0: "OK",
    -1: "E_INVAL invalid argument",
    -2: "E_NOMEM allocation failed",
    -3: "E_IO read failed",
    -4: "E_FORMAT bad magic/version",
    -5: "E_UNSUPPORTED not supported by this build",
    -6: "E_DEVICE CUDA error or device wait gave up",
}


def abi_available() -> bool:
    return _lib.LIB_PATH.exists()


def load_abi(force_rebuild: bool = False):
    return load_runtime(force_rebuild)


def status_str(code: int) -> str:
    return _STATUS_MSG.get(int(code), f"unknown status {code}")


def version() -> int:
    return int(load_abi().sn_abi_version())


def caps() -> int:
    return int(load_abi().sn_abi_caps())


def cap_names() -> list:
    m = caps()
    return [n for i, n in enumerate(CAPS) if m & (1 << i)]


def check(caller_major: int = ABI_MAJOR) -> int:
    return int(load_abi().sn_abi_check(int(caller_major)))


def _str(fn) -> str:
    n = fn(None, 0)
    buf = ctypes.create_string_buffer(n)
    fn(buf, n)
    return buf.value.decode()


def version_string() -> str:
    return _str(load_abi().sn_abi_version_string)


def backend_string() -> str:
    return _str(load_abi().sn_abi_backend_string)


class Rwkv7ABI:
    """Stable-ABI RWKV-7 handle (reference abi.py:152-189)."""

    def __init__(self, blob_path):
        self._lib = load_abi()
        self._h = self._lib.sn_abi_rwkv7_load(str(blob_path).encode())
        if not self._h:
            raise RuntimeError(f"sn_abi_rwkv7_load failed: {blob_path} ({_lib.last_error()})")
        self.vocab = int(self._lib.sn_abi_rwkv7_vocab(self._h))

    def reset(self):
        return int(self._lib.sn_abi_rwkv7_reset(self._h))

    def step(self, token: int) -> list:
        buf = (ctypes.c_float * self.vocab)()
        rc = int(self._lib.sn_abi_rwkv7_step(self._h, int(token), buf))
        if rc != STATUS_OK:
            raise RuntimeError(status_str(rc))
        return list(buf)

    def prefill(self, tokens) -> list:
        toks = list(tokens)
        ibuf = (ctypes.c_int32 * len(toks))(*toks)
        buf = (ctypes.c_float * self.vocab)()
        rc = int(self._lib.sn_abi_rwkv7_prefill(self._h, ibuf, len(toks), buf))
        if rc != STATUS_OK:
            raise RuntimeError(status_str(rc))
        return list(buf)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.sn_abi_rwkv7_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
