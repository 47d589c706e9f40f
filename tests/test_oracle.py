"""Pin the CPU oracle: against the committed golden vectors (made by the
reference itself, tests/golden/make_golden.py) and, where oracle/_ref is built,
against the reference runtime directly on fresh random inputs."""
from __future__ import annotations

import hashlib
import tempfile
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, rel_err
from sunnynet_b200 import formats

P = oracle.ptr


# ------------------------------------------------------------- primitives
@pytest.mark.parametrize("tag", ["a", "b", "c"])
@pytest.mark.parametrize("gated", [0, 1])
def test_scan_and_step_bit_exact_vs_golden(golden, tag, gated):
    g = golden("prims.npz")
    a, u, s0 = g[f"scan_{tag}_a"], g[f"scan_{tag}_u"], g[f"scan_{tag}_s0"]
    out, send = oracle.recur_scan(a, u, s0, gated)
    assert np.array_equal(out, g[f"scan_{tag}_g{gated}_out"])
    assert np.array_equal(send, g[f"scan_{tag}_g{gated}_send"])
    s = oracle.recur_step(np.ascontiguousarray(a[:, 0]), np.ascontiguousarray(u[:, 0]), s0, gated)
    assert np.array_equal(s, g[f"step_{tag}_g{gated}"])


@pytest.mark.parametrize("tag", ["a", "b"])
@pytest.mark.parametrize("gated", [0, 1])
def test_scan_bwd_bit_exact_vs_golden(golden, tag, gated):
    """sn_recur_bwd (recur.c:51-107) as the reference C computed it."""
    g = golden("prims.npz")
    a, u, s0 = g[f"bwd_{tag}_a"], g[f"bwd_{tag}_u"], g[f"bwd_{tag}_s0"]
    out, _ = oracle.recur_scan(a, u, s0, gated)
    assert np.array_equal(out, g[f"bwd_{tag}_g{gated}_out"])
    da, db, ds0 = oracle.recur_bwd(a, u, s0, out, g[f"bwd_{tag}_dout"], gated)
    assert np.array_equal(da, g[f"bwd_{tag}_g{gated}_da"])
    assert np.array_equal(db, g[f"bwd_{tag}_g{gated}_db"])
    assert np.array_equal(ds0, g[f"bwd_{tag}_g{gated}_ds0"])


@pytest.mark.parametrize("blk", [16, 0])
def test_quant_i8_bit_exact_vs_golden(golden, blk):
    g = golden("prims.npz")
    q, sc = oracle.quant_i8(g["q8_x"], blk)
    assert np.array_equal(q, g[f"q8_b{blk}_q"])
    assert np.array_equal(sc, g[f"q8_b{blk}_sc"])
    assert np.array_equal(oracle.dequant_i8(q, sc, blk), g[f"q8_b{blk}_xd"])


@pytest.mark.parametrize("blk", [64, 128])
def test_int4_and_w4a8_bit_exact_vs_golden(golden, blk):
    g = golden("prims.npz")
    W, x = g["q4_W"], g["q4_x"]
    q, sc = oracle.quant_i4(W, blk)
    assert np.array_equal(q, g[f"q4_b{blk}_q"]) and np.array_equal(sc, g[f"q4_b{blk}_sc"])
    assert np.array_equal(oracle.dequant_i4(q, sc, 256, blk), g[f"q4_b{blk}_wd"])
    assert np.array_equal(oracle.gemv_i4(x, q, sc, blk), g[f"q4_b{blk}_y"])
    # numpy quantiser used by the blob writer is the same arithmetic
    qn, scn = formats.quant_i4(W, blk)
    assert np.array_equal(qn, q) and np.array_equal(scn, sc)


def test_gemv_f32_bit_exact_vs_golden(golden):
    g = golden("prims.npz")
    y = np.empty(48, np.float32)
    x, W = g["q4_x"], g["q4_W"]  # keep the arrays alive across the call
    oracle.lib().or_gemv_f32(P(y), P(x), P(W), 256, 48)
    assert np.array_equal(y, g["gemv_f32_y"])


def test_w4a8_matches_explicit_integer_formula():
    """The reference's known-answer formula for the quantized path
    (tests/test_quant_i4.py:32-70), applied to the oracle."""
    rng = np.random.default_rng(1)
    out, n, block = 64, 256, 64
    W = rng.standard_normal((out, n)).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    q, s = oracle.quant_i4(W, block)
    half, nb = block // 2, n // block
    Wint = np.empty((out, n), np.int32)
    for b in range(nb):
        c = q[:, b * half:(b + 1) * half].astype(np.int32)
        Wint[:, b * block:b * block + half] = (c & 0x0F) - 8
        Wint[:, b * block + half:(b + 1) * block] = (c >> 4) - 8
    xq = np.empty(n, np.int8)
    xs = np.empty(nb, np.float32)
    for b in range(nb):
        seg = x[b * block:(b + 1) * block]
        amax = float(np.abs(seg).max())
        sc = amax / 127.0 if amax > 0 else 1.0
        xq[b * block:(b + 1) * block] = np.clip(np.rint(seg / sc), -127, 127).astype(np.int8)
        xs[b] = sc
    y_ref = np.zeros(out, np.float64)
    for b in range(nb):
        seg = slice(b * block, (b + 1) * block)
        y_ref += s[:, b] * xs[b] * (Wint[:, seg] * xq[seg].astype(np.int32)).sum(axis=1)
    y = oracle.gemv_i4(x, q, s, block)
    assert float(np.abs(y - y_ref).max()) < 1e-4


def test_int4_fp16_scale_roundtrip_bound():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((8, 256)) * 2.0).astype(np.float32)
    q, s = oracle.quant_i4(x, 128, fp16=True)
    qn, sn = formats.quant_i4(x, 128, fp16_scale=True)
    assert np.array_equal(q, qn) and np.array_equal(s.view(np.uint16), sn.view(np.uint16))
    xd = oracle.dequant_i4(q, s, 256, 128)
    assert np.array_equal(xd, formats.dequant_i4(qn, sn, 128))
    blk = s.astype(np.float32).reshape(8, 2)[:, :, None]
    assert np.all(np.abs(x - xd).reshape(8, 2, 128) <= blk / 2 + 1e-6)


# ------------------------------------------------------------- SunnyNet
def test_sunny_tiny_matches_reference_c_bit_exact(golden):
    g = golden("sunny_tiny.npz")
    m = oracle.Sunny(GOLDEN / "sunny_tiny.usnn", 1)
    lg = np.stack([m.step([t])[0] for t in g["tokens"]])
    assert np.array_equal(lg, g["logits_c"])
    assert rel_err(lg, g["logits_torch"]) < 1e-4
    assert np.array_equal(lg.argmax(1), g["logits_torch"].argmax(1))
    V, D, I, R, K, L = (int(v) for v in g["dims"])
    s, h = m.get_state(0, L, D, K - 1)
    assert rel_err(s, g["state_s"]) < 1e-4 and rel_err(h, g["state_hist"]) < 1e-4


def test_sunny_tiny_dbg_layer_bit_exact(golden):
    g = golden("sunny_tiny.npz")
    m = oracle.Sunny(GOLDEN / "sunny_tiny.usnn", 1)
    dbg = m.dbg_layer(int(g["dbg_tok"]), 1, g["dbg_layer1"].size)
    assert np.array_equal(dbg, g["dbg_layer1"])


def test_sunny_tiny_batched_matches_forward_step(golden):
    g = golden("sunny_tiny.npz")
    tb = g["tokens_b"]
    m = oracle.Sunny(GOLDEN / "sunny_tiny.usnn", tb.shape[0])
    for t in range(tb.shape[1]):
        lg = m.step(tb[:, t])
        assert rel_err(lg, g["logits_torch_b"][t]) < 1e-4
    V, D, I, R, K, L = (int(v) for v in g["dims"])
    for i in range(tb.shape[0]):
        s, h = m.get_state(i, L, D, K - 1)
        assert rel_err(s, g["final_s_b"][i]) < 1e-4
        assert rel_err(h, g["final_hist_b"][i]) < 1e-4


def test_sunny_tiny_stepwise_equals_chunked_forward(golden):
    """forward (chunked closed-form scan) == stepwise decode (test_architecture.py:357)."""
    g = golden("sunny_tiny.npz")
    idx = g["fwd_idx"]
    m = oracle.Sunny(GOLDEN / "sunny_tiny.usnn", idx.shape[0])
    for t in range(idx.shape[1]):
        lg = m.step(idx[:, t])
        if t % 7 == 0:
            assert rel_err(lg, g["fwd_logits"][:, t // 7]) < 1e-4
    assert rel_err(lg, g["fwd_logits_last"]) < 1e-4
    V, D, I, R, K, L = (int(v) for v in g["dims"])
    for i in range(idx.shape[0]):
        s, h = m.get_state(i, L, D, K - 1)
        # SunnyBlock.forward returns hist oldest-first (layers.py:266); the step
        # path and the C runtime keep it newest-first (layers.py:304,
        # sunnynet.c:234-237), which is the layout the state ABI uses.
        assert rel_err(s, g["fwd_s"][i]) < 1e-4
        assert rel_err(h, g["fwd_hist"][i][:, ::-1]) < 1e-4


def test_usnq_writer_deterministic(golden):
    """The INT8 blob written from the tiny model's weights is reproducible."""
    g = golden("sunny_tiny.npz")
    assert len(str(g["usnq_sha"])) == 64


# ------------------------------------------------------------- RWKV-7
def _rwkv_tiny_blobs(td: Path, golden):
    g = golden("rwkv_tiny.npz")
    L, D, HS, F, V, *ranks = (int(v) for v in g["shape"])
    shape = formats.RwkvShape(L, D, HS, F, V, tuple(ranks))
    w = formats.random_rwkv(shape, int(g["seed"]))
    paths = {}
    for kind in ("fp32", "q4", "q4g"):
        p = td / f"{kind}.bin"
        formats.write_krwk(p, w, quant=kind)
        paths[kind] = p
        assert hashlib.sha256(p.read_bytes()).hexdigest() == str(g[f"sha_{kind}"]), kind
    return g, shape, paths


def test_rwkv_tiny_matches_reference_c_bit_exact(golden):
    with tempfile.TemporaryDirectory() as td:
        g, shape, paths = _rwkv_tiny_blobs(Path(td), golden)
        for kind in ("fp32", "q4"):
            m = oracle.Rwkv(paths[kind], 1)
            lg = np.stack([m.step([t])[0] for t in g["tokens"]])
            assert np.array_equal(lg, g[f"logits_c_{kind}"]), kind
            m.reset()
            assert np.array_equal(m.dbg(int(g["tokens"][0]), 1, shape.dim), g[f"dbg_c_{kind}"])


def test_rwkv_tiny_fp32_matches_numpy_reference(golden):
    with tempfile.TemporaryDirectory() as td:
        g, shape, paths = _rwkv_tiny_blobs(Path(td), golden)
        m = oracle.Rwkv(paths["fp32"], 1)
        lg = np.stack([m.step([t])[0] for t in g["tokens"]])
        assert rel_err(lg, g["logits_numpy"]) < 1e-4
        assert np.array_equal(lg.argmax(1), g["logits_numpy"].argmax(1))
        S, sh = m.get_state(0, shape.layers, shape.n_head, shape.head_size, shape.dim)
        assert rel_err(S, g["S_numpy"]) < 1e-4 and rel_err(sh, g["shift_numpy"]) < 1e-4


def test_rwkv_tiny_q4g_tracks_reference_int4(golden):
    """Group-128 fp16-scale INT4 (no reference implementation) stays within the
    error of the reference's own block-64 INT4 format on the same model."""
    with tempfile.TemporaryDirectory() as td:
        g, shape, paths = _rwkv_tiny_blobs(Path(td), golden)
        ln = g["logits_numpy"]
        rel = {}
        for kind in ("q4", "q4g"):
            m = oracle.Rwkv(paths[kind], 1)
            lg = np.stack([m.step([t])[0] for t in g["tokens"]])
            rel[kind] = np.linalg.norm(lg - ln) / np.linalg.norm(ln)
        assert rel["q4g"] < 1.5 * rel["q4"], rel


def test_w4a8_g128_fp16_error_bound_vs_fp32():
    """GEMV-level INT4 error envelope of the reference (test_quant_i4.py:73-82)."""
    rng = np.random.default_rng(2)
    W = rng.standard_normal((256, 768)).astype(np.float32) * 0.05
    x = rng.standard_normal(768).astype(np.float32)
    q, s = oracle.quant_i4(W, 128, fp16=True)
    yq = oracle.gemv_i4(x, q, s, 128)
    yf = W @ x
    assert np.linalg.norm(yq - yf) / np.linalg.norm(yf) < 0.2


# ------------------------------------------- direct pin against oracle/_ref
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("B,T,N", [(1, 512, 1024), (2, 100, 77), (1, 33, 7)])
def test_scan_bit_exact_vs_ref_random(B, T, N):
    R = oracle.ref_abi()
    rng = np.random.default_rng(B * 1000 + N)
    H = np.exp(np.linspace(np.log(2), np.log(8192), N))
    a = rng.uniform(1 - 1 / H, 1.0, (B, T, N)).astype(np.float32)
    u = rng.standard_normal((B, T, N)).astype(np.float32)
    s0 = rng.standard_normal((B, N)).astype(np.float32)
    for gated in (0, 1):
        o = np.empty_like(a)
        se = np.empty((B, N), np.float32)
        R.sn_recur_scan(P(a), P(u), P(s0), P(o), P(se), B, T, N, gated)
        oo, ss = oracle.recur_scan(a, u, s0, gated)
        assert np.array_equal(o, oo) and np.array_equal(se, ss)


@needs_ref
@pytest.mark.parametrize("B,T,N", [(1, 512, 1024), (3, 70, 13)])
def test_scan_bwd_bit_exact_vs_ref_random(B, T, N):
    R = oracle.ref_abi()
    rng = np.random.default_rng(7 * B + N)
    H = np.exp(np.linspace(np.log(2), np.log(8192), N))
    a = rng.uniform(1 - 1 / H, 1.0, (B, T, N)).astype(np.float32)
    u = rng.standard_normal((B, T, N)).astype(np.float32)
    s0 = rng.standard_normal((B, N)).astype(np.float32)
    dout = rng.standard_normal((B, T, N)).astype(np.float32)
    for gated in (0, 1):
        out, _ = oracle.recur_scan(a, u, s0, gated)
        da, db = np.empty_like(a), np.empty_like(a)
        ds0 = np.empty((B, N), np.float32)
        R.sn_recur_bwd(P(a), P(u), P(s0), P(out), P(dout), P(da), P(db), P(ds0), B, T, N, gated)
        oa, ob, o0 = oracle.recur_bwd(a, u, s0, out, dout, gated)
        assert np.array_equal(da, oa) and np.array_equal(db, ob) and np.array_equal(ds0, o0)


@needs_ref
@pytest.mark.parametrize("out,n,block", [(300, 768, 64), (257, 768, 128), (64, 3072, 128)])
def test_w4a8_bit_exact_vs_ref_random(out, n, block):
    """fp16-scale INT4 codes widened to fp32 run through the reference
    sn_gemv_i4: the oracle's fp16-scale path must agree bit for bit."""
    R = oracle.ref_abi()
    rng = np.random.default_rng(out + n + block)
    W = (rng.standard_normal((out, n)) * 0.04).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    q, s16 = oracle.quant_i4(W, block, fp16=True)
    s32 = s16.astype(np.float32)
    y = np.empty(out, np.float32)
    R.sn_gemv_i4(P(y), P(x), P(q), P(s32), n, out, block)
    assert np.array_equal(oracle.gemv_i4(x, q, s16, block), y)
    assert np.array_equal(oracle.gemv_i4(x, q, s32, block), y)


@needs_ref
def test_sunny_random_preset_shape_bit_exact_vs_ref():
    """A perturbed random model with ragged sizes (dims not multiples of 8)."""
    R = oracle.ref_model()
    shape = formats.SunnyShape(1000, 72, 100, 36, 4, 3)
    w = formats.random_sunny(shape, seed=4, perturb=True)
    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "m.usnn"
        formats.write_usnn(p, w)
        h = R.sn_load(str(p).encode(), 1000, 72, 100, 36, 4, 3, 8, 1)
        assert h
        m = oracle.Sunny(p, 1)
        rng = np.random.default_rng(2)
        for t in rng.integers(0, 1000, 10):
            a = np.empty(1000, np.float32)
            R.sn_step(h, int(t), P(a))
            assert np.array_equal(m.step([t])[0], a)
        R.sn_free(h)


def test_rwkv_forced_step_fed_its_own_trace_equals_a_normal_step(golden):
    """The layer-by-layer checker: fed the residual stream a normal step
    produces, or_rk_step_forced reproduces that step bit for bit (logits and
    states). The trace is found by iterating the forced step from the same
    starting state until it is a fixed point: round k gets entries 0..k-1
    right, and the logits read entry L, so L+2 rounds."""
    g = golden("rwkv_tiny.npz")
    Lr, D, HS, F, V, *ranks = (int(v) for v in g["shape"])
    shape = formats.RwkvShape(Lr, D, HS, F, V, tuple(ranks))
    w = formats.random_rwkv(shape, int(g["seed"]))
    with tempfile.TemporaryDirectory() as td:
        for kind in ("fp32", "q4g"):
            p = Path(td) / f"{kind}.bin"
            formats.write_krwk(p, w, quant=kind)
            a, b = oracle.Rwkv(p, 3), oracle.Rwkv(p, 3)
            warm = np.array([5, 77, 300], np.int32)
            a.step(warm), b.step(warm)
            NH = D // HS
            st = [a.get_state(i, Lr, NH, HS, D) for i in range(3)]
            toks = np.array([9, 123, 400], np.int32)
            ref = a.step(toks)
            xs = np.zeros((3, Lr + 1, D), np.float32)
            for _ in range(Lr + 2):
                for i in range(3):
                    b.set_state(i, *st[i])
                xs, lg = b.step_forced(toks, xs)
            assert np.array_equal(lg, ref)
            for i in range(3):
                sa, ha = a.get_state(i, Lr, NH, HS, D)
                sb, hb = b.get_state(i, Lr, NH, HS, D)
                assert np.array_equal(sa, sb) and np.array_equal(ha, hb)


def test_sunny_row_parallel_equals_sequence_parallel():
    """With fewer sequences than threads the oracle runs them one at a time
    and spreads each GEMV's rows over the threads; the numbers must not move."""
    shape = formats.SunnyShape(700, 72, 100, 36, 4, 2)
    rng = np.random.default_rng(4)
    with tempfile.TemporaryDirectory() as td:
        p = Path(td) / "m.usnn"
        formats.write_usnn(p, formats.random_sunny(shape, seed=4, perturb=True))
        few, many = oracle.Sunny(p, 2), oracle.Sunny(p, 64)
        for _ in range(3):
            t = rng.integers(0, 700, 64).astype(np.int32)
            lm = many.step(t)
            lf = few.step(t[:2])
            assert np.array_equal(lf, lm[:2])


# ------------------------------------------ kernels module (sunnynet/kernels)
def _core_inputs(B, T, D, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, 2 * D)).astype(np.float32)
    H = np.exp(np.linspace(np.log(2.0), np.log(8192.0), D))
    delta = (1.0 / H).astype(np.float32)
    s0 = rng.standard_normal((B, D)).astype(np.float32)
    dstate = rng.standard_normal((B, T, D)).astype(np.float32)
    du = rng.standard_normal((B, T, D)).astype(np.float32)
    return q, delta, s0, dstate, du


needs_ref_kernels = pytest.mark.skipif(not oracle.REF_KERNELS_SO.exists(),
                                       reason="oracle/_ref kernels module not built")


@needs_ref_kernels
@pytest.mark.parametrize("B,T,D", [(1, 50, 16), (3, 33, 64), (2, 7, 40)])
def test_core_fwd_bwd_bit_exact_vs_reference_kernels(B, T, D):
    """core_fwd_f32 / core_bwd_f32 (core_avx2.c:34-148) and step_core_f32
    (step_avx2.c:54-86): the restatement is bit-identical (ddelta too: with
    one OpenMP thread the reference adds the sequences in order)."""
    R = oracle.ref_kernels()
    R.sn_set_threads(1)
    q, delta, s0, dstate, du = _core_inputs(B, T, D, B * 100 + D)
    st, u, p = (np.zeros((B, T, D), np.float32) for _ in range(3))
    R.core_fwd_f32(P(q), P(delta), P(s0), P(st), P(u), P(p), B, T, D)
    ost, ou, op = oracle.core_fwd(q, delta, s0)
    assert np.array_equal(st, ost) and np.array_equal(u, ou) and np.array_equal(p, op)
    dq = np.zeros_like(q)
    dd = np.zeros(D, np.float32)
    ds0 = np.zeros((B, D), np.float32)
    R.core_bwd_f32(P(q), P(delta), P(s0), P(st), P(u), P(p), P(dstate), P(du), P(dq), P(dd),
                   P(ds0), B, T, D)
    odq, odd, ods0 = oracle.core_bwd(q, delta, s0, st, u, p, dstate, du)
    assert np.array_equal(dq, odq) and np.array_equal(ds0, ods0) and np.array_equal(dd, odd)
    q1 = np.ascontiguousarray(q[:, 0])
    sn = np.zeros((B, D), np.float32)
    u1 = np.zeros((B, D), np.float32)
    R.step_core_f32(P(q1), P(delta), P(s0), P(sn), P(u1), B, D)
    ou1, osn = oracle.step_core(q1, delta, s0)
    assert np.array_equal(u1, ou1) and np.array_equal(sn, osn)
    assert np.array_equal(osn, ost[:, 0]) and np.array_equal(ou1, ou[:, 0])


@needs_ref_kernels
@pytest.mark.parametrize("B,D,taps", [(2, 64, 4), (3, 13, 4), (1, 40, 3)])
def test_dw_step_bit_exact_vs_reference_kernels(B, D, taps):
    R = oracle.ref_kernels()
    rng = np.random.default_rng(D)
    x = rng.standard_normal((B, D)).astype(np.float32)
    h = rng.standard_normal((B, taps - 1, D)).astype(np.float32)
    w = rng.standard_normal((taps, D)).astype(np.float32)
    acc = np.zeros((B, D), np.float32)
    R.dw_step_f32(P(x), P(h), P(w), P(acc), B, D, taps)
    assert np.array_equal(acc, oracle.dw_step(x, h, w))


@needs_ref_kernels
@pytest.mark.parametrize("B,T,N", [(2, 37, 13), (1, 300, 1024), (3, 20, 7)])
def test_kernels_scan_matches_recur_forms(B, T, N):
    """scan_f32 / scan_bwd_f32 (scan_avx2.c) are the gated recur_scan /
    recur_bwd with (a, u) = (p, nu); the module is GNU C, whose scalar tail
    (N % 8 channels) the compiler may contract: the oracle's gated scan must
    equal it on the vector channels, and its bwd everywhere."""
    R = oracle.ref_kernels()
    rng = np.random.default_rng(N)
    p = rng.uniform(0.3, 1.0, (B, T, N)).astype(np.float32)
    nu = rng.standard_normal((B, T, N)).astype(np.float32)
    s0 = rng.standard_normal((B, N)).astype(np.float32)
    out = np.zeros_like(p)
    se = np.zeros((B, N), np.float32)
    R.scan_f32(P(p), P(nu), P(s0), P(out), P(se), B, T, N)
    ro, rs = oracle.recur_scan(p, nu, s0, 1)
    nv = N - N % 8
    assert np.array_equal(out[..., :nv], ro[..., :nv])
    dout = rng.standard_normal((B, T, N)).astype(np.float32)
    dp, dn = np.zeros_like(p), np.zeros_like(p)
    d0 = np.zeros((B, N), np.float32)
    R.scan_bwd_f32(P(p), P(nu), P(s0), P(out), P(dout), P(dp), P(dn), P(d0), B, T, N)
    ra, rb, r0 = oracle.recur_bwd(p, nu, s0, out, dout, 1)
    assert np.array_equal(dp, ra) and np.array_equal(dn, rb) and np.array_equal(d0, r0)
    # every channel, the scalar tail included, follows the lane rule
    fo, fs = oracle.scan_f32(p, nu, s0)
    assert np.array_equal(out, fo) and np.array_equal(se, fs)
