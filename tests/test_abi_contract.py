"""C-ABI contract checks that need no GPU: the library loads, exports every
symbol include/*.h declares, and keeps the reference's version/caps/check/
string/thread semantics (reference tests/test_abi.py:28-48, 86-95)."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from conftest import REPO
from sunnynet_b200 import _lib


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from sunnynet_b200 import build
        build.build()
    return _lib.load()


def _declared_functions():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        txt = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        txt = re.sub(r"#.*", "", txt)
        for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", txt):
            n = m.group(1)
            if n.startswith("sn_") or n.endswith("_f32"):
                names.add(n)
    return names


def test_every_declared_symbol_is_exported(lib):
    declared = _declared_functions()
    assert len(declared) > 60
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared) <= set(_lib.SIGNATURES), set(declared) - set(_lib.SIGNATURES)


def test_version_and_strings(lib):
    assert lib.sn_abi_version() == 0x010100
    n = lib.sn_abi_version_string(None, 0)
    buf = ctypes.create_string_buffer(n)
    assert lib.sn_abi_version_string(buf, n) == n == 6
    assert buf.value == b"1.1.0"
    n = lib.sn_abi_backend_string(None, 0)
    buf = ctypes.create_string_buffer(n)
    lib.sn_abi_backend_string(buf, n)
    assert buf.value == b"cuda"
    # too-small buffer: returns the needed length, copies nothing
    small = ctypes.create_string_buffer(b"xx", 2)
    assert lib.sn_abi_backend_string(small, 2) == 5 and small.raw == b"xx"


def test_caps_superset_of_reference(lib):
    caps = lib.sn_abi_caps()
    for bit in range(5):  # RECUR_SCAN, RECUR_STEP, QUANT_I8, RWKV7, THREADS
        assert caps & (1 << bit)
    assert caps & (1 << 5)  # CUDA


def test_major_version_check(lib):
    assert lib.sn_abi_check(1) == 0
    assert lib.sn_abi_check(2) == -5
    assert lib.sn_abi_check(0) == -5


def test_threads_contract(lib):
    assert lib.sn_abi_set_threads(0) == -1
    assert lib.sn_abi_set_threads(-3) == -1
    assert lib.sn_abi_set_threads(6) == 0
    assert lib.sn_abi_get_threads() == 6
    assert lib.sn_recommended_threads() >= 1


def test_null_and_negative_dims_are_einval_without_device(lib):
    a = np.zeros((2, 8), np.float32)
    pa = _lib.ptr(a)
    assert lib.sn_abi_recur_step(None, pa, pa, 2, 8, 0) == -1
    assert lib.sn_abi_recur_step(pa, pa, pa, 2, -8, 0) == -1
    assert lib.sn_abi_recur_scan(pa, pa, pa, pa, pa, 2, -1, 8, 0) == -1
    assert lib.sn_abi_quant_i8(None, pa, pa, 2, 8, 0) == -1
    assert lib.sn_abi_dequant_i8(pa, pa, None, 2, 8, 0) == -1
    assert lib.sn_abi_rwkv7_step(None, 0, pa) == -1
    assert lib.sn_abi_rwkv7_prefill(None, pa, 1, pa) == -1
    assert lib.sn_abi_rwkv7_reset(None) == -1
    assert lib.sn_abi_rwkv7_vocab(None) == 0
    assert lib.sn_abi_rwkv7_load(None) is None
    assert lib.sn_abi_sunny_load(None, 1) is None
    assert lib.sn_abi_sunny_step(None, pa, 1, pa) == -1
    lib.sn_abi_rwkv7_free(None)
    lib.sn_abi_sunny_free(None)


def test_loaders_reject_bad_files_on_host(lib, tmp_path):
    """Header validation happens before any device work (sunnynet.c:363-368,
    rwkv7.c:419-422): missing file, wrong magic, truncated header."""
    assert lib.sn_abi_rwkv7_load(str(tmp_path / "nope.bin").encode()) is None
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"\x00" * 64)
    assert lib.sn_abi_rwkv7_load(str(bad).encode()) is None
    assert lib.sn_abi_sunny_load(str(bad).encode(), 1) is None
    assert lib.sn_load(str(bad).encode(), 16, 8, 8, 8, 4, 1, 8, 1) is None
    short = tmp_path / "short.bin"
    short.write_bytes(b"USNN")
    assert lib.sn_abi_sunny_load(str(short).encode(), 1) is None


# ------------------------------------------- the reference's own ctypes loaders
def _ref_bindings():
    import json
    from conftest import GOLDEN
    return json.loads((GOLDEN / "ref_bindings.json").read_text())


def test_reference_header_symbols_are_exported(lib):
    """Every function the reference's runtime headers declare (sn_abi.h,
    recur.h, quant.h, sunnynet.h, rwkv7.h), as recorded from the reference
    tree, is exported by this library."""
    heads = _ref_bindings()["headers"]
    want = sorted({n for names in heads.values() for n in names})
    assert "sn_recur_bwd" in want and len(want) >= 40
    missing = [n for n in want if not hasattr(lib, n)]
    assert not missing, missing


_KIND = {"void_p": "ptr", "float_p": "ptr", "char_p": "str", "int": "int", "uint32": "int",
         "int64": "int64", "void": "void"}


def _kind(t):
    if t is None:
        return "void"
    if t is ctypes.c_char_p:
        return "str"
    if t in (ctypes.c_void_p,) or (isinstance(t, type) and issubclass(t, ctypes._Pointer)):
        return "ptr"
    if t in (ctypes.c_int, ctypes.c_int32, ctypes.c_uint32):
        return "int"
    if t is ctypes.c_int64:
        return "int64"
    raise AssertionError(t)


def test_reference_loader_bindings_match_this_library(lib):
    """Each symbol the reference's loaders bind (runtime/__init__.py:135 binds
    sn_recur_bwd) exists here with the same number and kinds of arguments."""
    for loader, fns in _ref_bindings()["loaders"].items():
        for name, sig in fns.items():
            assert hasattr(lib, name), f"{loader} binds {name}, not exported"
            if name not in _lib.SIGNATURES:
                continue
            _, args = _lib.SIGNATURES[name]
            assert [_kind(t) for t in args] == [_KIND[t] for t in sig["argtypes"]], (loader, name)


def test_reference_loaders_run_against_this_library(monkeypatch):
    """The reference's own loader functions, with only the CDLL they open
    redirected to libsunnynet_cuda.so (the one-line change of the integration
    notes), set all their argtypes without an AttributeError."""
    import importlib
    import sys
    from conftest import REFERENCE_ROOT
    if not (REFERENCE_ROOT / "sunnynet" / "runtime" / "__init__.py").exists():
        pytest.skip("reference checkout not present")
    if not _lib.LIB_PATH.exists():
        from sunnynet_b200 import build
        build.build()
    monkeypatch.syspath_prepend(str(REFERENCE_ROOT))
    real = ctypes.CDLL
    monkeypatch.setattr(ctypes, "CDLL", lambda *a, **k: real(str(_lib.LIB_PATH)))
    loaders = {"__init__": "load_runtime", "model": "_load", "abi": "load_abi",
               "quant": "load_quant", "rwkv7_c": "_load", "kernels": "load_kernel"}
    try:
        for modname, fn in loaders.items():
            full = ("sunnynet.kernels" if modname == "kernels" else
                    "sunnynet.runtime" + ("" if modname == "__init__" else "." + modname))
            mod = importlib.import_module(full)
            for attr, val in (("_find_gcc", lambda: "gcc"), ("_needs_rebuild", lambda: False),
                              ("_lib", None)):
                if hasattr(mod, attr):
                    monkeypatch.setattr(mod, attr, val)
            handle = getattr(mod, fn)()
            assert handle is not None
            if modname == "__init__":
                assert handle.sn_recur_bwd.argtypes is not None
    finally:
        for name in list(sys.modules):
            if name == "sunnynet" or name.startswith("sunnynet."):
                sys.modules.pop(name)
