"""SunnyNet decode on the GPU vs the reference runtime and forward_step.

Tolerance (fp32 path): max|dlogit| <= 1e-4 * max|ref| per step (BASELINE
north_star: logits and states within 1e-4 relative), teacher-forced so one
near-tie cannot derail the comparison; argmax must match wherever the
reference's top-2 margin exceeds the tolerance. INT8 blobs (USNQ) are compared
with the oracle's W8A32 semantics (codes * row scale, then fp32) at the same
tolerance.
"""
from __future__ import annotations

import tempfile
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-4


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def check_logits(lg, ref, tol=TOL):
    lg = np.asarray(lg, np.float64).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    scale = np.abs(ref).max()
    err = np.abs(lg - ref).max()
    assert err <= tol * scale, f"max|d|={err:.3e} > {tol}*{scale:.3e}"
    for row_g, row_r in zip(lg, ref):
        a, b = int(row_g.argmax()), int(row_r.argmax())
        if a != b:
            top2 = np.sort(row_r)[-2:]
            margin = top2[1] - top2[0]
            assert margin <= 2 * tol * scale, f"argmax {a} != {b}, ref margin {margin:.3e}"


# ------------------------------------------------------ golden (reference-made)
def _golden_dims(g):
    V, D, I, R, K, L = (int(v) for v in g["dims"])
    return V, D, I, R, K, L


def test_internal_abi_matches_reference_c_and_torch(golden):
    from sunnynet_b200.runtime.model import SnModel
    g = golden("sunny_tiny.npz")
    V, D, I, R, K, L = _golden_dims(g)
    m = SnModel(GOLDEN / "sunny_tiny.usnn", V, D, I, R, K, L, 8, 1)
    for t, tok in enumerate(g["tokens"]):
        lg = np.array(m.step(int(tok)), np.float32)
        check_logits(lg, g["logits_c"][t])
        check_logits(lg, g["logits_torch"][t])


def test_prefill_equals_stepwise_and_reference(golden):
    """reference tests/test_runtime_model.py:41-58 (chunked prefill vs steps)."""
    from sunnynet_b200.runtime.model import SnModel
    g = golden("sunny_tiny.npz")
    V, D, I, R, K, L = _golden_dims(g)
    a = SnModel(GOLDEN / "sunny_tiny.usnn", V, D, I, R, K, L, 8, 1)
    lp = np.array(a.prefill([int(t) for t in g["tokens"]]), np.float32)
    b = SnModel(GOLDEN / "sunny_tiny.usnn", V, D, I, R, K, L, 8, 1)
    for t in g["tokens"]:
        last = np.array(b.step(int(t)), np.float32)
    check_logits(lp, last)
    check_logits(lp, g["prefill_logits_c"])
    # the state after the prefill continues exactly like the stepped one
    nxt = int(last.argmax())
    check_logits(np.array(a.step(nxt)), np.array(b.step(nxt)))


@pytest.mark.parametrize("chunk", [1, 7, 16, 40])
def test_chunked_prefill_matches_forward(golden, chunk):
    """Chunked prefill == SunnyNet.forward on the golden 2x40 prompt (final
    logits and state), for any chunk length (tests/test_architecture.py:127-161)."""
    from sunnynet_b200.model import SunnyBatch
    g = golden("sunny_tiny.npz")
    idx = g["fwd_idx"]
    m = SunnyBatch(GOLDEN / "sunny_tiny.usnn", idx.shape[0])
    lg = m.prefill(idx, chunk=chunk)
    check_logits(lg, g["fwd_logits_last"])
    s, h = m.get_state()
    assert rel_err(s, g["fwd_s"]) < TOL
    assert rel_err(h, g["fwd_hist"][:, :, ::-1]) < TOL


@pytest.mark.parametrize("B,T,chunk", [(3, 300, 64), (8, 512, 256)])
def test_chunked_prefill_vs_oracle_steps(B, T, chunk):
    """Random model: chunked prefill (tensor-core GEMMs over B*chunk rows +
    scan) vs the oracle stepping token by token; then decode continues."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(2000, 128, 224, 80, 4, 3)
    rng = np.random.default_rng(T)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, seed=2)
        toks = rng.integers(0, shape.vocab, (B, T)).astype(np.int32)
        gm, om = SunnyBatch(p, B), oracle.Sunny(p, B)
        lg = gm.prefill(toks, chunk=chunk)
        for t in range(T):
            ref = om.step(toks[:, t], want_logits=(t == T - 1))
        check_logits(lg, ref)
        s, h = gm.get_state()
        for i in range(B):
            rs, rh = om.get_state(i, shape.layers, shape.dim, shape.kh)
            assert rel_err(s[i], rs) < TOL and rel_err(h[i], rh) < TOL
        nxt = ref.argmax(1).astype(np.int32)
        check_logits(gm.step(nxt), om.step(nxt))


def test_dbg_layer_matches_reference(golden):
    from sunnynet_b200.runtime.model import SnModel
    g = golden("sunny_tiny.npz")
    V, D, I, R, K, L = _golden_dims(g)
    m = SnModel(GOLDEN / "sunny_tiny.usnn", V, D, I, R, K, L, 8, 1)
    ref = g["dbg_layer1"]
    dbg = np.array(m.dbg_layer(int(g["dbg_tok"]), 1, ref.size), np.float32)
    assert rel_err(dbg, ref) < TOL


def test_load_rejects_dims_mismatch(golden):
    from sunnynet_b200 import _lib
    lib = _lib.load()
    g = golden("sunny_tiny.npz")
    V, D, I, R, K, L = _golden_dims(g)
    p = str(GOLDEN / "sunny_tiny.usnn").encode()
    assert lib.sn_load(p, V, D, I, R, K, L + 1, 8, 1) is None
    assert lib.sn_load(p, V, D + 8, I, R, K, L, 8, 1) is None
    h = lib.sn_load(p, V, D, I, R, K, L, 8, 1)
    assert h and lib.sn_ready(h) == 1 and lib.sn_vocab(h) == V
    lib.sn_free(h)


def test_batched_matches_forward_step(golden):
    from sunnynet_b200.model import SunnyBatch
    g = golden("sunny_tiny.npz")
    tb = g["tokens_b"]
    m = SunnyBatch(GOLDEN / "sunny_tiny.usnn", tb.shape[0])
    for t in range(tb.shape[1]):
        check_logits(m.step(tb[:, t]), g["logits_torch_b"][t])
    s, h = m.get_state()
    assert rel_err(s, g["final_s_b"]) < TOL and rel_err(h, g["final_hist_b"]) < TOL


def test_stepwise_gpu_equals_chunked_forward(golden):
    """GPU stepwise decode over 40 tokens == SunnyNet.forward (chunked scan)."""
    from sunnynet_b200.model import SunnyBatch
    g = golden("sunny_tiny.npz")
    idx = g["fwd_idx"]
    m = SunnyBatch(GOLDEN / "sunny_tiny.usnn", idx.shape[0])
    for t in range(idx.shape[1]):
        lg = m.step(idx[:, t])
        if t % 7 == 0:
            check_logits(lg, g["fwd_logits"][:, t // 7])
    check_logits(lg, g["fwd_logits_last"])
    s, h = m.get_state()
    assert rel_err(s, g["fwd_s"]) < TOL
    assert rel_err(h, g["fwd_hist"][:, :, ::-1]) < TOL  # forward keeps hist oldest-first


# ------------------------------------------------------ random models vs oracle
def _blob(td, shape, quant=False, seed=0, fast=False):
    from sunnynet_b200 import formats
    w = formats.random_sunny(shape, seed=seed, perturb=True, fast=fast)
    p = Path(td) / ("m.usnq" if quant else "m.usnn")
    (formats.write_usnq if quant else formats.write_usnn)(p, w)
    return p


@pytest.mark.parametrize("B", [1, 3, 9, 70])
@pytest.mark.parametrize("quant", [False, True])
def test_random_model_vs_oracle(B, quant):
    """Ragged dims (D, I, R not multiples of 8/32), both weight formats, the
    GEMV path (B <= 8) and the tiled path (B > 8)."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(1000, 72, 100, 36, 4, 3)
    rng = np.random.default_rng(B)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, quant, seed=B)
        gm, om = SunnyBatch(p, B), oracle.Sunny(p, B)
        for _ in range(6):
            toks = rng.integers(0, 1000, B).astype(np.int32)
            check_logits(gm.step(toks), om.step(toks))
        s, h = gm.get_state()
        for i in range(B):
            rs, rh = om.get_state(i, 3, 72, 3)
            assert rel_err(s[i], rs) < TOL and rel_err(h[i], rh) < TOL


@pytest.mark.parametrize("B", [1, 4, 256])
def test_config2_shape_vs_oracle(B):
    """BASELINE config 2 (L4 d512 V16384, i896 r320), B=1/4/256."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SUNNY_PRESETS["c2"]
    rng = np.random.default_rng(0)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, seed=0, fast=True)
        gm, om = SunnyBatch(p, B), oracle.Sunny(p, B)
        for _ in range(3 if B > 8 else 6):
            toks = rng.integers(0, shape.vocab, B).astype(np.int32)
            check_logits(gm.step(toks), om.step(toks))


@pytest.mark.parametrize("B", [16, 64])
def test_config3_shape_int8_vs_oracle(B):
    """BASELINE config 3 (L12 d768 i1344 r480 V32000, INT8 per-row): the
    tensor-core path with exact bf16 INT8 codes (two MMAs per K step); r=480
    exercises a partial last K slab."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SUNNY_PRESETS["c3"]
    rng = np.random.default_rng(B)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, quant=True, seed=1, fast=True)
        gm, om = SunnyBatch(p, B), oracle.Sunny(p, B)
        for _ in range(2):
            toks = rng.integers(0, shape.vocab, B).astype(np.int32)
            check_logits(gm.step(toks), om.step(toks))


def test_state_export_import_roundtrip():
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(512, 64, 96, 32, 4, 2)
    rng = np.random.default_rng(3)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape)
        a = SunnyBatch(p, 2)
        for _ in range(5):
            a.step(rng.integers(0, 512, 2))
        s, h = a.get_state()
        b = SunnyBatch(p, 2)
        b.set_state(s, h)
        s2, h2 = b.get_state()
        assert np.array_equal(s, s2) and np.array_equal(h, h2)
        toks = rng.integers(0, 512, 2)
        assert np.array_equal(a.step(toks), b.step(toks))


def test_argmax_and_device_io():
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(2048, 64, 96, 32, 4, 2)
    rng = np.random.default_rng(4)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape)
        a, b = SunnyBatch(p, 16), SunnyBatch(p, 16)
        for _ in range(4):
            toks = rng.integers(0, 2048, 16).astype(np.int32)
            lg = a.step(toks)
            nx = b.step_argmax(torch.from_numpy(toks).cuda())
            assert np.array_equal(nx.cpu().numpy(), lg.argmax(1).astype(np.int32))


def test_half_weights_match_reference_half_runtime(golden):
    """sn_load_h against the reference's own fp16-weight runtime (sunnynet.c
    sn_load_h 459-578, gemv_h 142-167) on the same blob and tokens: the same
    five layer matrices and head rounded to fp16 (round to nearest even), so
    only the fp32 summation order differs: 1e-4 of max|ref| per step, while
    the half path itself sits ~7e-4 away from the fp32 runtime here."""
    from sunnynet_b200.runtime.model import SnModel
    g = golden("sunny_tiny.npz")
    V, D, I, R, K, L = _golden_dims(g)
    m = SnModel(GOLDEN / "sunny_tiny.usnn", V, D, I, R, K, L, 8, 1, half=True)
    for t, tok in enumerate(g["tokens"]):
        check_logits(np.array(m.step(int(tok)), np.float32), g["logits_c_half"][t])


def test_half_weights_track_fp32(golden):
    """sn_load_h (reference tests/test_runtime_model.py:123-167): bounded drift."""
    from sunnynet_b200.runtime.model import SnModel
    g = golden("sunny_tiny.npz")
    V, D, I, R, K, L = _golden_dims(g)
    a = SnModel(GOLDEN / "sunny_tiny.usnn", V, D, I, R, K, L, 8, 1)
    b = SnModel(GOLDEN / "sunny_tiny.usnn", V, D, I, R, K, L, 8, 1, half=True)
    worst = 0.0
    for t in g["tokens"]:
        la, lb = np.array(a.step(int(t))), np.array(b.step(int(t)))
        worst = max(worst, float(np.abs(la - lb).max()))
        assert np.isfinite(lb).all()
    assert worst < 2e-2


# --------------------------------------------- fused small-batch step (B <= 8)
def _steps(blob, B, toks_seq, fused):
    """Logits of each step and the final state, with the fused persistent step
    or the multi-kernel step (the fused one is taken for B <= 8 unless
    SN_DISABLE_FUSED is set; the library reads it at every step)."""
    import os
    from sunnynet_b200.model import SunnyBatch
    m = SunnyBatch(blob, B)
    old = os.environ.pop("SN_DISABLE_FUSED", None)
    try:
        if not fused:
            os.environ["SN_DISABLE_FUSED"] = "1"
        lgs = [m.step(t).copy() for t in toks_seq]
        s, h = m.get_state()
    finally:
        os.environ.pop("SN_DISABLE_FUSED", None)
        if old is not None:
            os.environ["SN_DISABLE_FUSED"] = old
    return lgs, s, h


@pytest.mark.parametrize("B", [1, 8])
@pytest.mark.parametrize("preset,quant", [("c2", False), ("mid", True), ("mid", False)])
def test_fused_step_matches_multi_kernel_step(B, preset, quant):
    """The one-kernel step (grid barriers between phases) against the
    multi-kernel step on the same tokens: logits and states within 1e-4."""
    from sunnynet_b200 import formats
    shape = (formats.SUNNY_PRESETS["c2"] if preset == "c2"
             else formats.SunnyShape(2000, 128, 224, 80, 4, 3))
    rng = np.random.default_rng(B + 10 * quant)
    toks = [rng.integers(0, shape.vocab, B).astype(np.int32) for _ in range(5)]
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, quant=quant, seed=2, fast=True)
        lf, sf, hf = _steps(p, B, toks, fused=True)
        lm, sm, hm = _steps(p, B, toks, fused=False)
    for a, b in zip(lf, lm):
        check_logits(a, b)
    assert rel_err(sf, sm) < TOL and rel_err(hf, hm) < TOL


def test_config3_shape_int8_fused_vs_oracle():
    """BASELINE config 3 shape (INT8 per-row) at B=2: the fused step's int8
    weight rows against the oracle."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SUNNY_PRESETS["c3"]
    rng = np.random.default_rng(7)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, quant=True, seed=1, fast=True)
        gm, om = SunnyBatch(p, 2), oracle.Sunny(p, 2)
        for _ in range(3):
            toks = rng.integers(0, shape.vocab, 2).astype(np.int32)
            check_logits(gm.step(toks), om.step(toks))


@pytest.mark.parametrize("B", [2, 16])
def test_bad_token_id_is_reported_and_handle_stays_usable(B):
    """A token id outside the vocabulary is never read from the table: the
    step reports SN_E_DEVICE (the device-side index check) and the next step
    with valid ids runs normally (fused path at B=2, multi-kernel at B=16)."""
    from sunnynet_b200 import formats
    from sunnynet_b200._lib import SnError
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(512, 64, 96, 32, 4, 2)
    rng = np.random.default_rng(5)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape)
        m = SunnyBatch(p, B)
        bad = rng.integers(0, 512, B).astype(np.int32)
        bad[B // 2] = 512 + 7
        with pytest.raises(SnError) as ei:
            m.step(bad)
        assert ei.value.code == -6
        m.reset()
        om = oracle.Sunny(p, B)
        for _ in range(3):
            toks = rng.integers(0, 512, B).astype(np.int32)
            check_logits(m.step(toks), om.step(toks))


@pytest.mark.parametrize("B", [1, 3, 8])
def test_fused_argmax_matches_logits_in_place(B):
    """Greedy steps of the fused path write the argmax straight into the
    caller's device buffer, which here also holds the input tokens (as a decode
    loop does): each step's ids must equal the argmax of the logits of a twin
    model fed the same tokens (lowest id on ties)."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(2048, 64, 96, 32, 4, 2)
    rng = np.random.default_rng(11 + B)
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape)
        a, b = SunnyBatch(p, B), SunnyBatch(p, B)
        cur = torch.from_numpy(rng.integers(0, 2048, B).astype(np.int32)).cuda()
        for _ in range(5):
            toks = cur.cpu().numpy().copy()
            lg = a.step(toks)
            b.step_argmax(cur, out=cur)
            torch.cuda.synchronize()
            assert np.array_equal(cur.cpu().numpy(), lg.argmax(1).astype(np.int32))


# ------------------------------- batched tensor-core step: planes + side stream
@pytest.mark.parametrize("B", [16, 40, 130])
@pytest.mark.parametrize("quant", [False, True])
def test_tc_step_planes_equal_split_step(B, quant):
    """The tensor-core step whose producers write the bf16 input planes (and
    whose feedback contractions run on a side stream) against the same
    contractions fed by a split launch each (SN_TC_SPLIT_STEP, read at load):
    the planes hold the same values, so logits and states are bit-identical."""
    import os
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(2000, 128, 224, 80, 4, 3)
    rng = np.random.default_rng(B)
    toks = [rng.integers(0, shape.vocab, B).astype(np.int32) for _ in range(4)]
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, quant=quant, seed=5, fast=True)
        a = SunnyBatch(p, B)
        os.environ["SN_TC_SPLIT_STEP"] = "1"
        try:
            b = SunnyBatch(p, B)
        finally:
            os.environ.pop("SN_TC_SPLIT_STEP", None)
        om = oracle.Sunny(p, B)
        for t in toks:
            la, lb = a.step(t), b.step(t)
            assert np.array_equal(la, lb)
            check_logits(la, om.step(t))
        sa, ha = a.get_state()
        sb, hb = b.get_state()
        assert np.array_equal(sa, sb) and np.array_equal(ha, hb)


@pytest.mark.parametrize("quant", [False, True])
def test_split_k_cluster_matches_unsplit_and_oracle(quant):
    """Few-tile contractions split K over a thread-block cluster (partials
    summed across the cluster's shared memory in rank order). Against the
    same model with the split off (SN_TC_NO_SPLITK, read when a step is
    captured) and against the oracle: both within the fp32 tolerance, and the
    split path is deterministic (two models, identical logits)."""
    import os
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    # K = 512 / 640: 8 and 10 slabs, enough for the split (Ws, V, Wz, Wc)
    shape = formats.SunnyShape(3000, 512, 640, 160, 4, 2)
    B = 48
    rng = np.random.default_rng(7 + quant)
    toks = [rng.integers(0, shape.vocab, B).astype(np.int32) for _ in range(3)]
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, quant=quant, seed=8, fast=True)
        a, a2 = SunnyBatch(p, B), SunnyBatch(p, B)
        os.environ["SN_TC_NO_SPLITK"] = "1"
        try:
            b = SunnyBatch(p, B)
            lb = [b.step(t) for t in toks]
        finally:
            os.environ.pop("SN_TC_NO_SPLITK", None)
        om = oracle.Sunny(p, B)
        for t, l_b in zip(toks, lb):
            la = a.step(t)
            assert np.array_equal(la, a2.step(t))
            ref = om.step(t)
            check_logits(la, ref)
            check_logits(l_b, ref)


@pytest.mark.parametrize("mode", [1, 2])
def test_profile_modes_report_families_and_leave_results_alone(mode):
    """Kernel-family timing: mode 1 runs the step kernel by kernel, mode 2
    replays an instrumented copy of the step's graph. Either way the logits
    and states equal those of an unprofiled model, and every contraction
    family of the tensor-core step is reported once per layer and step."""
    from sunnynet_b200 import _lib, formats
    from sunnynet_b200.model import SunnyBatch
    shape = formats.SunnyShape(2000, 128, 224, 80, 4, 3)
    B = 32
    rng = np.random.default_rng(40 + mode)
    toks = [rng.integers(0, shape.vocab, B).astype(np.int32) for _ in range(3)]
    lib = _lib.load()
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, seed=4, fast=True)
        a, b = SunnyBatch(p, B), SunnyBatch(p, B)
        la = [a.step(t).copy() for t in toks]
        _lib.check(lib.sn_abi_cuda_profile(mode))
        try:
            lb = [b.step(t).copy() for t in toks]
        finally:
            _lib.check(lib.sn_abi_cuda_profile(0))
        rep = _lib.profile_report()
    for x, y in zip(la, lb):
        assert np.array_equal(x, y)
    for fam in ("gemm_V", "gemm_U", "gemm_Wz", "gemm_Wc", "gemm_Ws"):
        n, ms = rep[fam]
        assert n == 3 * shape.layers and ms > 0, (fam, rep[fam])
    assert rep["gemm_head"][0] == 3


def test_batch_engine_matches_requests_served_alone():
    """Continuous batching on the GPU: 7 requests of different prompt lengths
    and budgets through 3 slots (admission, slot reuse, state hand-off from
    the prefill handle) against each request decoded alone on a one-sequence
    handle, teacher-forced with the engine's own tokens: every logits row
    within the fp32 tolerance."""
    from sunnynet_b200 import formats
    from sunnynet_b200.model import SunnyBatch
    from sunnynet_b200.serve import BatchEngine
    shape = formats.SunnyShape(1500, 128, 224, 80, 4, 3)
    rng = np.random.default_rng(21)
    specs = [(5, 6), (9, 4), (9, 8), (17, 5), (3, 10), (30, 3), (9, 7)]
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, seed=21)
        eng = BatchEngine(p, slots=3, prefill_chunk=8)
        reqs = [eng.submit(list(rng.integers(0, shape.vocab, n)), m, record_logits=True)
                for n, m in specs]
        eng.run()
        alone = SunnyBatch(p, 1)
        for r in reqs:
            assert r.done and len(r.tokens) == r.max_tokens
            alone.reset()
            ref = alone.prefill(np.array([r.prompt], np.int32), chunk=8)
            for k, tok in enumerate(r.tokens):
                check_logits(r.logits[k], ref)
                assert tok == int(np.argmax(r.logits[k]))
                if k + 1 < len(r.tokens):
                    ref = alone.step(np.array([tok], np.int32))
    # greedy requests without recorded logits take the device argmax path
    with tempfile.TemporaryDirectory() as td:
        p = _blob(td, shape, seed=21)
        a, b = BatchEngine(p, slots=3, prefill_chunk=8), BatchEngine(p, slots=3, prefill_chunk=8)
        prompts = [list(rng.integers(0, shape.vocab, n)) for n in (4, 7, 7, 12)]
        ra = [a.submit(q, 6) for q in prompts]
        rb = [b.submit(q, 6, record_logits=True) for q in prompts]
        a.run(), b.run()
        for x, y in zip(ra, rb):
            assert x.tokens == y.tokens
