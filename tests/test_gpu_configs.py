"""Parity at the shapes and batch sizes the benchmark runs (BASELINE configs
2-5), through the C-ABI, against the CPU oracle.

fp32 (and INT8 W8A32) paths: logits within 1e-4 of max|ref| per step,
teacher-forced (both sides get the same token ids), argmax equal unless the
reference's top-2 margin is inside that tolerance; recurrent states within 1e-4
relative. Where the oracle would need minutes for every sequence of a large
batch, the GPU still runs the whole batch and the oracle follows a strided
subset of its sequences (rows are independent, so each checked row is a full
parity check of that row).

RWKV-7 at the config-4 shape is checked layer by layer: the GPU step reports
the residual stream entering each layer, the oracle runs every layer from that
same input (and from the GPU's state at the start of the step), so each
layer's output and state carry only that layer's kernel error rather than the
random 12-layer model's amplification of it. Bounds: 1e-4 with fp32 weights
(every fp32 operation of the same kernels at the same shapes). With INT4
group-128 W4A8 weights the integer block dot products are identical (bit-exact
GEMV tests), but each of the layer's ~10 activation vectors is quantised to
INT8 per 128-block from fp32 values that differ in the last bits (summation
order, libm vs CUDA exp/tanh); a value on a rounding boundary quantises one
code apart, moving that block's products by one activation step (amax/127 of
the block), and such flips feed the heads' group norm and the next
projections inside the same layer. Bound 2e-2 of the row's max per layer
(logits and states alike); the observed distribution is printed.
"""
from __future__ import annotations

import os
import tempfile
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import rel_err
from test_gpu_sunny import check_logits

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-4
TOL_Q4 = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _sunny_blob(td, shape, quant=False, seed=0):
    from sunnynet_b200 import formats
    w = formats.random_sunny(shape, seed=seed, perturb=True, fast=True)
    p = Path(td) / ("m.usnq" if quant else "m.usnn")
    (formats.write_usnq if quant else formats.write_usnn)(p, w)
    return p


def _check_states(gs, gh, om, rows, shape):
    for j, i in enumerate(rows):
        rs, rh = om.get_state(j, shape.layers, shape.dim, shape.kh)
        assert rel_err(gs[i], rs) < TOL, (i, rel_err(gs[i], rs))
        assert rel_err(gh[i], rh) < TOL, (i, rel_err(gh[i], rh))


# ---------------------------------------------------------------- config 3
def test_config3_b1024_int8_from_warm_states():
    """Config 3 (L12 d768 i1344 r480 V32000, INT8 per-output-row) at its
    benchmarked batch, B=1024 on one GPU: the tile widths and K splits the
    cost model picks at M=1024. Both sides start from the same non-zero
    states (imported), then 4 teacher-forced steps; every row is checked."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SUNNY_PRESETS["c3"]
    B = 1024
    rng = np.random.default_rng(31)
    s0 = (0.5 * rng.standard_normal((B, shape.layers, shape.dim))).astype(np.float32)
    h0 = rng.standard_normal((B, shape.layers, shape.kh, shape.dim)).astype(np.float32)
    with tempfile.TemporaryDirectory() as td:
        p = _sunny_blob(td, shape, quant=True, seed=3)
        gm, om = SunnyBatch(p, B), oracle.Sunny(p, B)
        gm.set_state(s0, h0)
        for i in range(B):
            om.set_state(i, s0[i], h0[i])
        for _ in range(4):
            toks = rng.integers(0, shape.vocab, B).astype(np.int32)
            check_logits(gm.step(toks), om.step(toks))
        gs, gh = gm.get_state()
        _check_states(gs, gh, om, range(B), shape)


def test_config3_int8_codes_converted_in_mainloop_match_planes():
    """INT8 dequant inside the contraction's main loop (converter warps turn
    each K slab of 1-byte codes into the bf16 slab the MMAs read) against the
    default load-time bf16 code planes: the tensor cores see the same operand
    values, so logits and states are bit-identical. Config-3 shape at
    B=1024 (the benchmarked tile widths and K splits)."""
    from sunnynet_b200 import _lib, formats
    from sunnynet_b200.model import SunnyBatch
    lib = _lib.load()
    shape = formats.SUNNY_PRESETS["c3"]
    B = 1024
    rng = np.random.default_rng(33)
    s0 = (0.5 * rng.standard_normal((B, shape.layers, shape.dim))).astype(np.float32)
    h0 = rng.standard_normal((B, shape.layers, shape.kh, shape.dim)).astype(np.float32)
    toks = [rng.integers(0, shape.vocab, B).astype(np.int32) for _ in range(3)]
    out = []
    with tempfile.TemporaryDirectory() as td:
        p = _sunny_blob(td, shape, quant=True, seed=5)
        for mode in (0, 1):
            old = lib.sn_abi_cuda_int8_mainloop(mode)
            try:
                gm = SunnyBatch(p, B)  # weights prepared under this setting
            finally:
                lib.sn_abi_cuda_int8_mainloop(old)
            gm.set_state(s0, h0)
            logits = [gm.step(t).copy() for t in toks]
            out.append((logits, gm.get_state()))
            gm.close()
    (la, (sa, ha)), (lb, (sb, hb)) = out
    for x, y in zip(la, lb):
        assert np.array_equal(x, y)
    assert np.array_equal(sa, sb) and np.array_equal(ha, hb)


# ---------------------------------------------------------------- config 2
def test_config2_b256_prefill_then_256_decode_steps():
    """Config 2 (L4 d512 V16384, fp32 weights on the bf16x3 tensor-core path)
    at B=256 over the config's whole run: a 256-token chunked prefill, then
    256 teacher-forced decode steps, so any drift of the split-precision
    contractions would accumulate in the states. The oracle follows every
    8th sequence; logits are compared after the prefill and every 32 steps,
    states at the end."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SUNNY_PRESETS["c2"]
    B, T, steps = 256, 256, 256
    rows = list(range(0, B, 8))
    rng = np.random.default_rng(2)
    prompt = rng.integers(0, shape.vocab, (B, T)).astype(np.int32)
    with tempfile.TemporaryDirectory() as td:
        p = _sunny_blob(td, shape, seed=0)
        gm, om = SunnyBatch(p, B), oracle.Sunny(p, len(rows))
        lg = gm.prefill(prompt, chunk=256)
        for t in range(T):
            ref = om.step(prompt[rows, t], want_logits=(t == T - 1))
        check_logits(lg[rows], ref)
        for k in range(steps):
            toks = rng.integers(0, shape.vocab, B).astype(np.int32)
            want = k % 32 == 31
            lg = gm.step(toks)
            ref = om.step(toks[rows], want_logits=want)
            if want:
                check_logits(lg[rows], ref)
        gs, gh = gm.get_state()
        _check_states(gs, gh, om, rows, shape)


# ---------------------------------------------------------------- config 5
def test_config5_width_picks_192_column_tile():
    """The config-5 widths (d1536 i2688 r960 V32000) at 2048 prefill rows per
    chunk (8 sequences x 256): M=2048, N=K=1536 is where the tile cost model
    picks the 192-column tile for the feedback contraction (one wave of 128
    tiles instead of two of 192 at BN=128). Two layers, not 24: every
    contraction has the config's shape; the oracle steps 2048 tokens. Chunked
    prefill (scan ring sized to the chunk) vs stepping: last logits and the
    final (s, hist)."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(32000, 1536, 2688, 960, 4, 2)
    B, T = 8, 256
    rng = np.random.default_rng(5)
    toks = rng.integers(0, shape.vocab, (B, T)).astype(np.int32)
    with tempfile.TemporaryDirectory() as td:
        p = _sunny_blob(td, shape, seed=5)
        gm, om = SunnyBatch(p, B), oracle.Sunny(p, B)
        lg = gm.prefill(toks, chunk=256)
        for t in range(T):
            ref = om.step(toks[:, t], want_logits=(t == T - 1))
        check_logits(lg, ref)
        gs, gh = gm.get_state()
        _check_states(gs, gh, om, range(B), shape)


def test_config5_full_depth_two_chunks_final_state():
    """Config 5 itself (L24 d1536 i2688 r960 V32000, fp32): 2 sequences of
    512 tokens as two 256-token chunks carrying only (s, hist), against the
    oracle stepping token by token: final states within 1e-4, last logits."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SUNNY_PRESETS["c5"]
    B, T = 2, 512
    rng = np.random.default_rng(55)
    toks = rng.integers(0, shape.vocab, (B, T)).astype(np.int32)
    with tempfile.TemporaryDirectory() as td:
        p = _sunny_blob(td, shape, seed=55)
        gm, om = SunnyBatch(p, B), oracle.Sunny(p, B)
        lg = gm.prefill(toks, chunk=256)
        for t in range(T):
            ref = om.step(toks[:, t], want_logits=(t == T - 1))
        check_logits(lg, ref)
        gs, gh = gm.get_state()
        _check_states(gs, gh, om, range(B), shape)


@pytest.mark.parametrize("quant", [False, True])
def test_forced_192_column_tile_at_small_batch(quant):
    """The 192-column tile forced on every contraction that may take it
    (SN_TC_FORCE_BN, read when a step is captured) on a decode step at B=48,
    against the oracle; INT8 weights never take it, so that case checks the
    hook leaves them on their own widths."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(3000, 768, 1344, 480, 4, 2)
    B = 48
    rng = np.random.default_rng(9 + quant)
    prompt = rng.integers(0, shape.vocab, (B, 64)).astype(np.int32)
    with tempfile.TemporaryDirectory() as td:
        p = _sunny_blob(td, shape, quant=quant, seed=9)
        om = oracle.Sunny(p, B)
        os.environ["SN_TC_FORCE_BN"] = "192"
        try:
            gm = SunnyBatch(p, B)
            for _ in range(3):
                toks = rng.integers(0, shape.vocab, B).astype(np.int32)
                check_logits(gm.step(toks), om.step(toks))
            lg = gm.prefill(prompt, chunk=64)  # 3072 rows per chunk
        finally:
            os.environ.pop("SN_TC_FORCE_BN", None)
        for t in range(prompt.shape[1]):
            ref = om.step(prompt[:, t], want_logits=(t == prompt.shape[1] - 1))
        check_logits(lg, ref)
        gs, gh = gm.get_state()
        _check_states(gs, gh, om, range(B), shape)


# ---------------------------------------------------------------- config 4
@pytest.fixture(scope="module")
def c4_blobs():
    from sunnynet_b200 import formats
    shape = formats.RWKV_PRESETS["c4"]
    w = formats.random_rwkv(shape, 0)
    td = tempfile.mkdtemp()
    p32, p4 = Path(td) / "c4.f32.bin", Path(td) / "c4.q4g.bin"
    formats.write_krwk(p32, w, quant="fp32")
    formats.write_krwk(p4, w, quant="q4g", group=128)
    return shape, {"fp32": p32, "q4g": p4}


def _row_rel(a, b):
    """max over rows of max|a-b| / max|b| (rows along the last axis)."""
    a = np.asarray(a, np.float64).reshape(-1, a.shape[-1])
    b = np.asarray(b, np.float64).reshape(-1, b.shape[-1])
    return float((np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)).max())


@pytest.mark.parametrize("B", [64, 512])
@pytest.mark.parametrize("kind", ["fp32", "q4g"])
def test_config4_layer_by_layer_teacher_forced(c4_blobs, B, kind):
    """Config 4 (RWKV-7 L12 D768 H12x64 F3072 V65536) at B=64 and B=512 on
    one GPU. Two free steps give every sequence a non-zero state; then, for
    two steps, the oracle takes the GPU's states (every 16th sequence), the
    GPU step reports each layer's input, and the oracle runs each layer from
    that input: every layer's output, the logits from the GPU's last layer
    output, and every layer's new state are compared."""
    from sunnynet_b200.rwkv7 import Rwkv7Batch
    shape, paths = c4_blobs
    tol = TOL if kind == "fp32" else TOL_Q4
    rows = list(range(0, B, 16))
    L, NH, HS, D = shape.layers, shape.n_head, shape.head_size, shape.dim
    gm, om = Rwkv7Batch(paths[kind], B), oracle.Rwkv(paths[kind], len(rows))
    rng = np.random.default_rng(B + (kind == "q4g"))
    for _ in range(2):
        gm.step(rng.integers(0, shape.vocab, B).astype(np.int32))
    for _ in range(2):
        S, sh = gm.get_state()
        for j, i in enumerate(rows):
            om.set_state(j, S[i], sh[i])
        toks = rng.integers(0, shape.vocab, B).astype(np.int32)
        lg, xs = gm.step_trace(toks)
        xo, lo = om.step_forced(toks[rows], xs[rows])
        errs = [_row_rel(xs[rows, l], xo[:, l]) for l in range(L + 1)]
        print(f"{kind} B={B} per-layer max row error:", " ".join(f"{e:.1e}" for e in errs))
        for l, err in enumerate(errs):
            assert err < tol, (kind, B, "layer output", l, err)
        err = _row_rel(lg[rows], lo)
        assert err < tol, (kind, B, "logits", err)
        S2, sh2 = gm.get_state()
        for j, i in enumerate(rows):
            rS, rsh = om.get_state(j, L, NH, HS, D)
            for l in range(L):
                assert rel_err(S2[i, l], rS[l]) < tol, (kind, B, "state", i, l)
                assert rel_err(sh2[i, l], rsh[l]) < tol, (kind, B, "shift", i, l)
