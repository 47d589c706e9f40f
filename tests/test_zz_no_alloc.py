"""sn_abi_recur_scan_noalloc against the regular scan entry point.

The no-allocation entry point is for callers that cannot let the library
call cudaMalloc/cudaFree: a process whose device memory belongs to its own
pool allocator, a loop that must not stall on the device synchronisation
those calls imply, a fixed memory budget. Its temporary chunk records live in
a fixed 2 MiB device array instead of growing library scratch, so it accepts
B*N <= 262144 and device arrays only.

Its arithmetic is scan mode 1 of sn_abi_recur_scan (per-chunk affine maps
composed into each chunk's carry), so it is checked against the regular entry
point in both modes with the chunked-scan tolerance of the other scan tests:
1e-4 relative to the largest state of each channel. Two calls in a row with
different shapes show that what the first call leaves in the shared array
does not leak into the second.

This file is collected last, so a run that stops at its first failure has
already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TOL = 1e-4  # the chunked-scan tolerance of the scan tests
CAP = 1 << 18  # channels (B*N) the fixed scratch holds


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from sunnynet_b200 import _lib, runtime
    runtime.load_runtime()
    return runtime, _lib


def _inputs(B, T, N, seed):
    rng = np.random.default_rng(seed)
    H = np.exp(np.linspace(np.log(2.0), np.log(8192.0), N))
    a = rng.uniform(1.0 - 1.0 / H, 1.0, (B, T, N)).astype(np.float32)
    u = rng.standard_normal((B, T, N)).astype(np.float32)
    s0 = rng.standard_normal((B, N)).astype(np.float32)
    return [torch.from_numpy(x).cuda() for x in (a, u, s0)]


def _noalloc(lib, da, du, ds, gated):
    from sunnynet_b200._lib import check, ptr
    B, T, N = da.shape
    out = torch.empty_like(da)
    send = torch.empty_like(ds)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib.load().sn_abi_recur_scan_noalloc(ptr(da), ptr(du), ptr(ds), ptr(out), ptr(send),
                                                B, T, N, gated, stream),
          "recur_scan_noalloc")
    torch.cuda.synchronize()
    return out.cpu().numpy(), send.cpu().numpy()


def _regular(runtime, da, du, ds, gated, mode):
    old = runtime.set_scan_mode(mode)
    try:
        out, send = runtime.scan(da, du, ds, gated=bool(gated))
    finally:
        runtime.set_scan_mode(old)
    torch.cuda.synchronize()
    return out.cpu().numpy(), send.cpu().numpy()


def _assert_close(out, send, ref_out, ref_send):
    scale = np.maximum(np.abs(ref_out.astype(np.float64)).max(axis=1, keepdims=True), 1e-30)
    assert float((np.abs(out.astype(np.float64) - ref_out) / scale).max()) < TOL
    sscale = np.maximum(np.abs(ref_out.astype(np.float64)).max(axis=1), 1e-30)
    assert float((np.abs(send.astype(np.float64) - ref_send) / sscale).max()) < TOL
    assert np.array_equal(send, out[:, -1])


def test_two_calls_in_a_row_match_the_regular_entry_point(env):
    runtime, lib = env
    # a large call, then a smaller one of another shape and form: the second
    # reads nothing the first left behind
    for (B, T, N, gated, seed) in [(1, 4096, 1024, 1, 0), (3, 777, 40, 0, 1)]:
        da, du, ds = _inputs(B, T, N, seed)
        out, send = _noalloc(lib, da, du, ds, gated)
        for mode in (1, 0):  # chunked, and the bit-exact sequential scan
            ref_out, ref_send = _regular(runtime, da, du, ds, gated, mode)
            _assert_close(out, send, ref_out, ref_send)


def test_repeated_calls_give_the_same_result(env):
    runtime, lib = env
    da, du, ds = _inputs(2, 1000, 36, 2)
    first = _noalloc(lib, da, du, ds, 1)
    second = _noalloc(lib, da, du, ds, 1)
    assert np.array_equal(first[0], second[0])
    assert np.array_equal(first[1], second[1])


def test_rejects_sizes_beyond_the_fixed_scratch(env):
    _, lib = env
    from sunnynet_b200._lib import ptr
    L = lib.load()
    x = torch.zeros(4, device="cuda")
    p = ptr(x)
    rc = L.sn_abi_recur_scan_noalloc(p, p, p, p, p, 2, 4, CAP // 2 + 1, 1, None)
    assert rc == -1  # SN_E_INVAL, nothing launched
    assert "fixed scratch" in lib.last_error()


def test_rejects_host_arrays(env):
    _, lib = env
    from sunnynet_b200._lib import ptr
    a = np.zeros((1, 8, 4), np.float32)
    s = np.zeros((1, 4), np.float32)
    o = np.zeros_like(a)
    e = np.zeros_like(s)
    rc = lib.load().sn_abi_recur_scan_noalloc(ptr(a), ptr(a), ptr(s), ptr(o), ptr(e), 1, 8, 4, 1,
                                              None)
    assert rc == -1
    assert "device memory" in lib.last_error()


_FRESH = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, {repo!r})
import oracle
from sunnynet_b200 import _lib
L = _lib.load()  # only the no-allocation entry point is called below
rng = np.random.default_rng(5)
B, T, N = 2, 600, 256
H = np.exp(np.linspace(np.log(2.0), np.log(8192.0), N))
a = rng.uniform(1.0 - 1.0 / H, 1.0, (B, T, N)).astype(np.float32)
u = rng.standard_normal((B, T, N)).astype(np.float32)
s0 = rng.standard_normal((B, N)).astype(np.float32)
da, du, ds = (torch.from_numpy(x).cuda() for x in (a, u, s0))
for call in range(2):
    out = torch.full_like(da, float("nan"))
    send = torch.full_like(ds, float("nan"))
    rc = L.sn_abi_recur_scan_noalloc(_lib.ptr(da), _lib.ptr(du), _lib.ptr(ds), _lib.ptr(out),
                                     _lib.ptr(send), B, T, N, 1, None)
    assert rc == 0, (rc, _lib.last_error())
    torch.cuda.synchronize()
    ro, rs = oracle.recur_scan(a, u, s0, 1)
    o, s = out.cpu().numpy().astype(np.float64), send.cpu().numpy().astype(np.float64)
    scale = np.maximum(np.abs(ro.astype(np.float64)).max(axis=1, keepdims=True), 1e-30)
    err = float((np.abs(o - ro) / scale).max())
    assert err < {tol}, err
    assert np.array_equal(send.cpu().numpy(), out.cpu().numpy()[:, -1])
print("fresh-process no-alloc scan ok")
"""


def test_fresh_process_calls_only_the_no_alloc_entry_point():
    """The intended use: a process that never lets the library initialise its
    runtime (no stream, no mapped error word, no scratch) and calls only this
    entry point, twice, on torch-allocated device arrays; checked against the
    CPU oracle's recurrence (the reference's per-row rule)."""
    import subprocess
    import sys

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from conftest import REPO
    code = _FRESH.format(repo=str(REPO), tol=TOL)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       timeout=600, cwd=str(REPO))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "fresh-process no-alloc scan ok" in r.stdout


def test_rejects_arrays_of_another_device(env):
    """Arrays must live on the current device: another GPU's arrays would be
    read across NVLink (or fault without peer access), so they are refused
    before anything is launched."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _, lib = env
    from sunnynet_b200._lib import ptr
    other = torch.zeros(64, device="cuda:1")
    mine = torch.zeros(64, device="cuda:0")
    with torch.cuda.device(0):
        rc = lib.load().sn_abi_recur_scan_noalloc(ptr(other), ptr(mine), ptr(mine), ptr(mine),
                                                  ptr(mine), 1, 8, 8, 1, None)
    assert rc == -1
    assert "current device" in lib.last_error()
