"""The kernels module on the GPU (scan_f32, scan_bwd_f32, core_fwd_f32,
core_bwd_f32, step_core_f32, dw_step_f32) against the CPU oracle, whose
restatements are pinned bit for bit to the reference's own kernels library
(tests/test_oracle.py); and the autograd operators against torch autograd of
the same math in float64.

Bars: scan_f32, scan_bwd_f32 and dw_step_f32 bit-exact. The core functions
round every operation as the reference except exp (CUDA expf vs the host
libm, a couple of ulp): forward outputs within 1e-5 of max|ref| per array,
backward within 1e-4 (the delta gradient sums T*B terms).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from sunnynet_b200 import _lib, kernels
    kernels.load_kernel()
    return _lib


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _core_inputs(B, T, D, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, 2 * D)).astype(np.float32)
    H = np.exp(np.linspace(np.log(2.0), np.log(8192.0), D))
    delta = (1.0 / H).astype(np.float32)
    s0 = rng.standard_normal((B, D)).astype(np.float32)
    dstate = rng.standard_normal((B, T, D)).astype(np.float32)
    du = rng.standard_normal((B, T, D)).astype(np.float32)
    return q, delta, s0, dstate, du


def _call(lib, name, *args):
    L = lib.load()
    L.sn_abi_clear_error()
    getattr(L, name)(*[lib.ptr(a) if hasattr(a, "shape") else a for a in args])
    assert lib.last_error() == "", lib.last_error()


@pytest.mark.parametrize("B,T,N", [(2, 37, 13), (1, 4096, 1024), (3, 65, 40)])
@pytest.mark.parametrize("device", [False, True])
def test_scan_f32_and_bwd_bit_exact(lib, B, T, N, device):
    rng = np.random.default_rng(N + device)
    p = rng.uniform(0.3, 1.0, (B, T, N)).astype(np.float32)
    nu = rng.standard_normal((B, T, N)).astype(np.float32)
    s0 = rng.standard_normal((B, N)).astype(np.float32)
    dout = rng.standard_normal((B, T, N)).astype(np.float32)
    ro, rs = oracle.scan_f32(p, nu, s0)
    ra, rb, r0 = oracle.recur_bwd(p, nu, s0, ro, dout, 1)
    conv = (lambda x: torch.from_numpy(x).cuda()) if device else (lambda x: x)
    back = (lambda x: x.cpu().numpy()) if device else (lambda x: x)
    P_, U_, S_, D_ = conv(p), conv(nu), conv(s0), conv(dout)
    out, send = conv(np.zeros_like(p)), conv(np.zeros((B, N), np.float32))
    _call(lib, "scan_f32", P_, U_, S_, out, send, B, T, N)
    torch.cuda.synchronize()
    assert np.array_equal(back(out), ro) and np.array_equal(back(send), rs)
    dp, dn, d0 = conv(np.zeros_like(p)), conv(np.zeros_like(p)), conv(np.zeros((B, N), np.float32))
    _call(lib, "scan_bwd_f32", P_, U_, S_, conv(ro), D_, dp, dn, d0, B, T, N)
    torch.cuda.synchronize()
    assert np.array_equal(back(dp), ra) and np.array_equal(back(dn), rb)
    assert np.array_equal(back(d0), r0)


@pytest.mark.parametrize("B,T,D", [(1, 50, 16), (3, 33, 64), (2, 700, 512), (2, 9, 13)])
def test_core_fwd_bwd_and_step_vs_oracle(lib, B, T, D):
    q, delta, s0, dstate, du = _core_inputs(B, T, D, B * 7 + D)
    ost, ou, op = oracle.core_fwd(q, delta, s0)
    DV = D - D % 8
    nan = np.float32("nan")
    st, u, p = (np.full((B, T, D), nan, np.float32) for _ in range(3))
    _call(lib, "core_fwd_f32", q, delta, s0, st, u, p, B, T, D)
    for g, r in ((st, ost), (u, ou), (p, op)):
        assert _rel(g[..., :DV], r[..., :DV]) < 1e-5
        assert np.isnan(g[..., DV:]).all()  # the partial group is left untouched
    # backward from the same forward outputs, so only the reverse pass differs
    rdq, rdd, rds0 = oracle.core_bwd(q, delta, s0, ost, ou, op, dstate, du)
    dq = np.full_like(q, nan)
    dd = np.zeros(D, np.float32)
    ds0 = np.full((B, D), nan, np.float32)
    _call(lib, "core_bwd_f32", q, delta, s0, ost, ou, op, dstate, du, dq, dd, ds0, B, T, D)
    dqv = dq.reshape(B, T, 2, D)[..., :DV]
    rqv = rdq.reshape(B, T, 2, D)[..., :DV]
    assert _rel(dqv, rqv) < 1e-4
    assert _rel(ds0[:, :DV], rds0[:, :DV]) < 1e-4
    assert _rel(dd[:DV], rdd[:DV]) < 1e-4
    # ddelta accumulates into what the caller passes
    dd2 = np.full(D, 1.0, np.float32)
    _call(lib, "core_bwd_f32", q, delta, s0, ost, ou, op, dstate, du, dq, dd2, ds0, B, T, D)
    assert _rel(dd2[:DV] - 1.0, rdd[:DV]) < 1e-4
    # one decode step = the first row of the forward pass
    q1 = np.ascontiguousarray(q[:, 0])
    sn, u1 = np.zeros((B, D), np.float32), np.zeros((B, D), np.float32)
    _call(lib, "step_core_f32", q1, delta, s0, sn, u1, B, D)
    ru1, rsn = oracle.step_core(q1, delta, s0)
    assert _rel(sn[:, :DV], rsn[:, :DV]) < 1e-5 and _rel(u1[:, :DV], ru1[:, :DV]) < 1e-5


@pytest.mark.parametrize("B,D,taps", [(2, 64, 4), (3, 13, 4), (5, 40, 3), (1, 8, 1)])
def test_dw_step_bit_exact(lib, B, D, taps):
    rng = np.random.default_rng(D + taps)
    x = rng.standard_normal((B, D)).astype(np.float32)
    h = rng.standard_normal((B, max(taps - 1, 1), D)).astype(np.float32)
    w = rng.standard_normal((taps, D)).astype(np.float32)
    acc = np.zeros((B, D), np.float32)
    _call(lib, "dw_step_f32", x, h, w, acc, B, D, taps)
    assert np.array_equal(acc, oracle.dw_step(x, h[:, :taps - 1].copy(), w))


def _torch_core(q, delta, s0):
    """The fused core written with torch ops (float64): competition over
    groups of 8 (rolls -1 / -2), decay gate, scan."""
    B, T, D2 = q.shape
    D = D2 // 2
    ur, g = q[..., :D], q[..., D:]
    gg = g.reshape(B, T, D // 8, 8)
    w = (torch.sigmoid(gg - torch.roll(gg, -1, dims=-1)) *
         torch.sigmoid(gg - torch.roll(gg, -2, dims=-1))).reshape(B, T, D)
    u = ur * w
    p = 1.0 - delta * (1.0 - torch.sigmoid(g))
    s, states = s0, []
    for t in range(T):
        s = p[:, t] * s + (1.0 - p[:, t]) * u[:, t]
        states.append(s)
    return u, torch.stack(states, 1)


def test_core_autograd_matches_torch_float64(lib):
    from sunnynet_b200 import kernels
    B, T, D = 2, 40, 32
    q, delta, s0, dstate, du = _core_inputs(B, T, D, 11)
    args = [torch.from_numpy(x).cuda().requires_grad_() for x in (q, delta, s0)]
    u, st = kernels.core_forward(*args)
    (torch.from_numpy(du).cuda() * u).sum().backward(retain_graph=True)
    (torch.from_numpy(dstate).cuda() * st).sum().backward()
    ref = [torch.from_numpy(x).cuda().double().requires_grad_() for x in (q, delta, s0)]
    ru, rst = _torch_core(*ref)
    ((torch.from_numpy(du).cuda().double() * ru).sum() +
     (torch.from_numpy(dstate).cuda().double() * rst).sum()).backward()
    assert _rel(u.detach().cpu(), ru.detach().cpu()) < 1e-5
    assert _rel(st.detach().cpu(), rst.detach().cpu()) < 1e-5
    for a, r in zip(args, ref):
        assert _rel(a.grad.cpu(), r.grad.cpu()) < 1e-4


def test_scan_autograd_matches_torch_float64(lib):
    from sunnynet_b200 import kernels
    B, T, N = 3, 100, 24
    rng = np.random.default_rng(5)
    u = rng.standard_normal((B, T, N)).astype(np.float32)
    p = rng.uniform(0.5, 1.0, (B, T, N)).astype(np.float32)
    s0 = rng.standard_normal((B, N)).astype(np.float32)
    w = rng.standard_normal((B, T, N)).astype(np.float32)
    args = [torch.from_numpy(x).cuda().requires_grad_() for x in (u, p, s0)]
    states, last = kernels.scan_auto(*args)
    (torch.from_numpy(w).cuda() * states).sum().backward()
    ref = [torch.from_numpy(x).cuda().double().requires_grad_() for x in (u, p, s0)]
    s, out = ref[2], []
    for t in range(T):
        s = ref[1][:, t] * s + (1.0 - ref[1][:, t]) * ref[0][:, t]
        out.append(s)
    rs = torch.stack(out, 1)
    (torch.from_numpy(w).cuda().double() * rs).sum().backward()
    assert _rel(states.detach().cpu(), rs.detach().cpu()) < 1e-5
    assert torch.equal(last, states[:, -1])
    for a, r in zip(args, ref):
        assert _rel(a.grad.cpu(), r.grad.cpu()) < 1e-4


def test_reference_kernels_loader_bindings_drive_this_library(lib, golden):
    """The argtypes the reference's kernels/__init__.py load_kernel sets
    (recorded in the committed fixture), applied to a fresh handle of this
    library, then one call of each symbol."""
    import ctypes
    import json
    from conftest import GOLDEN
    sigs = json.loads((GOLDEN / "ref_bindings.json").read_text())["loaders"][
        "kernels/__init__.py:load_kernel"]
    h = ctypes.CDLL(str(lib.LIB_PATH))
    kinds = {"void_p": ctypes.c_void_p, "int": ctypes.c_int}
    for name, sig in sigs.items():
        getattr(h, name).argtypes = [kinds[t] for t in sig["argtypes"]]
    B, T, D = 2, 16, 16
    q, delta, s0, dstate, du = _core_inputs(B, T, D, 3)
    P = lambda a: a.ctypes.data  # noqa: E731
    st, u, p = (np.zeros((B, T, D), np.float32) for _ in range(3))
    h.core_fwd_f32(P(q), P(delta), P(s0), P(st), P(u), P(p), B, T, D)
    ost, _, _ = oracle.core_fwd(q, delta, s0)
    assert _rel(st, ost) < 1e-5
    out, send = np.zeros_like(st), np.zeros((B, D), np.float32)
    h.scan_f32(P(p), P(u), P(s0), P(out), P(send), B, T, D)
    assert np.array_equal(out, oracle.scan_f32(p, u, s0)[0])
    h.sn_set_threads(4)
