"""Generate the committed golden fixtures from the reference itself.

Runs only where the reference tree exists (it imports the reference's Python
package and loads the reference C runtime built by oracle/Makefile into
oracle/_ref). Outputs small files into tests/golden/; the tests then need
neither the reference tree nor oracle/_ref.

    python tests/golden/make_golden.py --ref <reference checkout>

What is pinned:
* prims.npz      -- sn_recur_scan/step/bwd, sn_quant_i8/dequant_i8, sn_quant_i4/
                    dequant_i4, sn_gemv_i4, sn_gemv_f32 outputs of the reference C
                    on seeded inputs (ragged sizes included).
* sunny_tiny.*   -- a tiny SunnyNet built by the reference's torch code
                    (SunnyNet(SunnyConfig) with perturbed norms), exported by the
                    reference's release.export_runtime_blob; logits of the
                    reference C runtime (sn_step) and of SunnyNet.forward_step,
                    batched forward_step, chunked forward (prefill) final state,
                    and an sn_dbg_layer dump.
* ref_bindings.json -- every symbol the reference's ctypes loaders bind, with
                    the argtypes/restype they set, and the functions its
                    runtime headers declare (the drop-in boundary).
* rwkv_tiny.npz  -- a tiny RWKV-7 drawn by sunnynet_b200.formats.random_rwkv,
                    written to GGUF, run through the reference numpy RWKV7.step,
                    exported by the reference's _export_rwkv7.py (fp32 and INT4)
                    and run through the reference C sn_rk_step; plus sha256 of
                    the reference-exported blobs (our writer must reproduce them).
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

import oracle  # noqa: E402
from sunnynet_b200 import formats  # noqa: E402

P = oracle.ptr


def sha(path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


# ------------------------------------------------------------------ primitives
def make_prims(out: Path):
    R = oracle.ref_abi()
    rng = np.random.default_rng(1234)
    d = {}
    for tag, (B, T, N) in {"a": (2, 37, 13), "b": (1, 64, 40), "c": (3, 5, 8)}.items():
        a = rng.uniform(0.3, 1.0, (B, T, N)).astype(np.float32)
        u = rng.standard_normal((B, T, N)).astype(np.float32)
        s0 = rng.standard_normal((B, N)).astype(np.float32)
        for g in (0, 1):
            o = np.empty_like(a)
            se = np.empty((B, N), np.float32)
            R.sn_recur_scan(P(a), P(u), P(s0), P(o), P(se), B, T, N, g)
            d[f"scan_{tag}_g{g}_out"], d[f"scan_{tag}_g{g}_send"] = o, se
            s = s0.copy()
            a0, u0 = np.ascontiguousarray(a[:, 0]), np.ascontiguousarray(u[:, 0])
            R.sn_recur_step(P(a0), P(u0), P(s), B, N, g)
            d[f"step_{tag}_g{g}"] = s
        d[f"scan_{tag}_a"], d[f"scan_{tag}_u"], d[f"scan_{tag}_s0"] = a, u, s0
    # INT8 per-block quant, ragged last block, a zero block
    x = rng.standard_normal((3, 70)).astype(np.float32) * 3
    x[1, 16:32] = 0.0
    for blk in (16, 0):
        nb = (70 + blk - 1) // blk if blk > 0 else 1
        q = np.empty((3, 70), np.int8)
        sc = np.empty((3, nb), np.float32)
        R.sn_quant_i8(P(x), P(q), P(sc), 3, 70, blk)
        xd = np.empty((3, 70), np.float32)
        R.sn_dequant_i8(P(q), P(sc), P(xd), 3, 70, blk)
        d[f"q8_b{blk}_q"], d[f"q8_b{blk}_sc"], d[f"q8_b{blk}_xd"] = q, sc, xd
    d["q8_x"] = x
    # INT4 + W4A8 GEMV, blocks 64 and 128, with a zero group
    W = (rng.standard_normal((48, 256)) * 0.05).astype(np.float32)
    W[3, :64] = 0.0
    xv = rng.standard_normal(256).astype(np.float32)
    for blk in (64, 128):
        q = np.empty((48, 128), np.uint8)
        sc = np.empty((48, 256 // blk), np.float32)
        R.sn_quant_i4(P(W), P(q), P(sc), 48, 256, blk)
        wd = np.empty((48, 256), np.float32)
        R.sn_dequant_i4(P(q), P(sc), P(wd), 48, 256, blk)
        y = np.empty(48, np.float32)
        R.sn_gemv_i4(P(y), P(xv), P(q), P(sc), 256, 48, blk)
        d[f"q4_b{blk}_q"], d[f"q4_b{blk}_sc"], d[f"q4_b{blk}_wd"], d[f"q4_b{blk}_y"] = q, sc, wd, y
    yf = np.empty(48, np.float32)
    R.sn_gemv_f32(P(yf), P(xv), P(W), 256, 48)
    d["q4_W"], d["q4_x"], d["gemv_f32_y"] = W, xv, yf
    # sn_recur_bwd (recur.c:51-107): reverse pass over the forward scan's
    # outputs, both forms, ragged N (the AVX2 lanes and the scalar tail)
    for tag, (B, T, N) in {"a": (2, 37, 13), "b": (1, 64, 40)}.items():
        a = rng.uniform(0.3, 1.0, (B, T, N)).astype(np.float32)
        u = rng.standard_normal((B, T, N)).astype(np.float32)
        s0 = rng.standard_normal((B, N)).astype(np.float32)
        dout = rng.standard_normal((B, T, N)).astype(np.float32)
        d[f"bwd_{tag}_a"], d[f"bwd_{tag}_u"], d[f"bwd_{tag}_s0"] = a, u, s0
        d[f"bwd_{tag}_dout"] = dout
        for g in (0, 1):
            o = np.empty_like(a)
            se = np.empty((B, N), np.float32)
            R.sn_recur_scan(P(a), P(u), P(s0), P(o), P(se), B, T, N, g)
            da, db = np.empty_like(a), np.empty_like(a)
            ds0 = np.empty((B, N), np.float32)
            R.sn_recur_bwd(P(a), P(u), P(s0), P(o), P(dout), P(da), P(db), P(ds0), B, T, N, g)
            d[f"bwd_{tag}_g{g}_out"] = o
            d[f"bwd_{tag}_g{g}_da"], d[f"bwd_{tag}_g{g}_db"] = da, db
            d[f"bwd_{tag}_g{g}_ds0"] = ds0
    np.savez_compressed(out / "prims.npz", **d)


# -------------------------------------------------------------------- SunnyNet
def make_sunny(out: Path, ref_root: Path):
    import torch
    sys.path.insert(0, str(ref_root))
    from sunnynet.model import SunnyConfig, SunnyNet
    from sunnynet import release

    torch.manual_seed(0)
    cfg = SunnyConfig(vocab_size=512, dim=64, inner=96, rank=32, taps=4, layers=2,
                      h_max=8192.0, scan_chunk=16)
    m = SunnyNet(cfg)
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        for blk in m.blocks:
            for nm in (blk.norm_in, blk.norm_mix):
                nm.gamma.add_(0.1 * torch.randn(nm.gamma.shape, generator=g))
                nm.center.add_(0.05 * torch.randn(nm.center.shape, generator=g))
            blk.a.fill_(0.8)
            blk.b_gain.fill_(0.35)
            blk.circ.t.copy_(torch.tensor([0.2, 0.55, 0.3]))
            blk.theta.add_(0.3 * torch.randn(blk.theta.shape, generator=g))
        m.norm_out.gamma.add_(0.1 * torch.randn(cfg.dim, generator=g))
        m.norm_out.center.add_(0.05 * torch.randn(cfg.dim, generator=g))
    m.eval()
    with tempfile.TemporaryDirectory() as td:
        ck = Path(td) / "tiny.pt"
        torch.save({"arch": "sunnynet", "config": cfg.__dict__, "model": m.state_dict(),
                    "summary": {}}, ck)
        blob = out / "sunny_tiny.usnn"
        release.export_runtime_blob(ck, blob)

    # our writer must reproduce the reference exporter byte for byte
    S = formats.SunnyShape(cfg.vocab_size, cfg.dim, cfg.inner, cfg.rank, cfg.taps, cfg.layers)
    w = formats.SunnyWeights(shape=S)
    for blk in m.blocks:
        Wm = blk.W_s.weight
        t0, t1, t2 = blk.circ.t[0], blk.circ.t[1], blk.circ.t[2]
        ws = (t0 * torch.roll(Wm, -1, dims=1) + t1 * Wm + t2 * torch.roll(Wm, 1, dims=1))
        w.layers.append({
            "ni_g": blk.norm_in.gamma.detach().numpy(), "ni_c": blk.norm_in.center.detach().numpy(),
            "nm_g": blk.norm_mix.gamma.detach().numpy(), "nm_c": blk.norm_mix.center.detach().numpy(),
            "dw": blk.dw.weight.detach().reshape(cfg.dim, cfg.taps).numpy(),
            "V": blk.V.weight.detach().numpy(), "U": blk.U.weight.detach().numpy(),
            "Wz": blk.W_z.weight.detach().numpy(), "Wc": blk.W_c.weight.detach().numpy(),
            "Ws_eff": ws.detach().numpy(), "delta": blk.delta().detach().numpy(),
            "a_tanh": float(torch.tanh(blk.a.detach())), "b_gain": float(blk.b_gain.detach())})
    w.no_g = m.norm_out.gamma.detach().numpy()
    w.no_c = m.norm_out.center.detach().numpy()
    w.embed = m.embed.weight.detach().numpy()
    with tempfile.TemporaryDirectory() as td:
        mine = Path(td) / "mine.usnn"
        formats.write_usnn(mine, w)
        assert mine.read_bytes() == blob.read_bytes(), "write_usnn differs from release.py"
        minq = Path(td) / "mine.usnq"
        formats.write_usnq(minq, w)
        qsha = sha(minq)

    V = cfg.vocab_size
    tg = torch.Generator().manual_seed(7)
    toks = torch.randint(0, V, (24,), generator=tg)
    # reference C runtime, B=1
    RM = oracle.ref_model()
    h = RM.sn_load(str(blob).encode(), V, cfg.dim, cfg.inner, cfg.rank, cfg.taps, cfg.layers, 8, 1)
    assert h, "reference sn_load failed"
    lc = np.empty((24, V), np.float32)
    for t in range(24):
        RM.sn_step(h, int(toks[t]), P(lc[t]))
    # prefill of the same 24 tokens on a fresh state returns the last logits
    RM.sn_reset(h)
    tk = np.ascontiguousarray(toks.numpy().astype(np.int32))
    lp = np.empty(V, np.float32)
    RM.sn_prefill(h, P(tk), 24, P(lp))
    # per-layer dump: fresh state, token toks[0], layer 1
    RM.sn_reset(h)
    # raw, at, v, gate, u, s, zn, yn, sfb, out (sunnynet.c:278-290)
    ndbg = 7 * cfg.dim + cfg.rank + 2 * cfg.inner
    dbg = np.zeros(ndbg, np.float32)
    RM.sn_dbg_layer(h, int(toks[0]), 1, P(dbg))
    RM.sn_free(h)
    # the reference's fp16-weight runtime (sn_load_h / gemv_h, sunnynet.c:142-167,
    # 459-578) on the same blob and tokens; every row length here is a
    # multiple of 16, so gemv_h never reaches its scalar tail
    hh = RM.sn_load_h(str(blob).encode(), V, cfg.dim, cfg.inner, cfg.rank, cfg.taps,
                      cfg.layers, 8, 1)
    assert hh, "reference sn_load_h failed"
    lch = np.empty((24, V), np.float32)
    for t in range(24):
        RM.sn_step(hh, int(toks[t]), P(lch[t]))
    RM.sn_free(hh)

    with torch.no_grad():
        st = m.init_state(1)
        lt = []
        for t in range(24):
            lg, st = m.forward_step(toks[t:t + 1], st)
            lt.append(lg[0].numpy())
        lt = np.stack(lt)
        s1, h1 = st.s[0].numpy(), st.hist[0].numpy()
        # batched teacher-forced decode, B=3
        tb = torch.randint(0, V, (3, 12), generator=tg)
        stb = m.init_state(3)
        lb = []
        for t in range(12):
            lg, stb = m.forward_step(tb[:, t], stb)
            lb.append(lg.numpy())
        lb = np.stack(lb)
        # chunked prefill (SunnyNet.forward with carried state), B=2, T=40 in 2 segments
        idx = torch.randint(0, V, (2, 40), generator=tg)
        s0 = m.init_state(2)
        o1, s_mid = m(idx[:, :25], s0, return_state=True)
        o2, s_end = m(idx[:, 25:], s_mid, return_state=True)
        fwd_logits = torch.cat([o1, o2], dim=1).numpy()
    np.savez_compressed(
        out / "sunny_tiny.npz",
        dims=np.array([V, cfg.dim, cfg.inner, cfg.rank, cfg.taps, cfg.layers], np.int32),
        tokens=toks.numpy().astype(np.int32), logits_c=lc, logits_torch=lt,
        logits_c_half=lch,
        prefill_logits_c=lp, dbg_tok=np.int32(toks[0]), dbg_layer1=dbg,
        state_s=s1, state_hist=h1,
        tokens_b=tb.numpy().astype(np.int32), logits_torch_b=lb,
        final_s_b=stb.s.numpy(), final_hist_b=stb.hist.numpy(),
        fwd_idx=idx.numpy().astype(np.int32), fwd_logits_last=fwd_logits[:, -1],
        fwd_logits=fwd_logits[:, ::7], fwd_s=s_end.s.numpy(), fwd_hist=s_end.hist.numpy(),
        usnq_sha=np.array(qsha))


# ---------------------------------------------------------------------- RWKV-7
def _write_gguf(path: Path, w: formats.RwkvWeights):
    import gguf
    S = w.shape
    wr = gguf.GGUFWriter(str(path), arch="rwkv7")
    wr.add_uint32("rwkv7.block_count", S.layers)
    wr.add_uint32("rwkv7.embedding_length", S.dim)
    wr.add_uint32("rwkv7.wkv.head_size", S.head_size)
    wr.add_uint32("rwkv7.feed_forward_length", S.ffn)
    wr.add_float32("rwkv7.attention.layer_norm_epsilon", w.eps)
    wr.add_array("tokenizer.ggml.tokens", [f"t{i}" for i in range(S.vocab)])
    t = lambda n, a: wr.add_tensor(n, np.ascontiguousarray(a, np.float32))
    t("token_embd.weight", w.embed)
    t("token_embd_norm.weight", w.en_w)
    t("token_embd_norm.bias", w.en_b)
    for i, ly in enumerate(w.layers):
        p = f"blk.{i}."
        t(p + "attn_norm.weight", ly["ln1w"]); t(p + "attn_norm.bias", ly["ln1b"])
        t(p + "attn_norm_2.weight", ly["ln2w"]); t(p + "attn_norm_2.bias", ly["ln2b"])
        t(p + "time_mix_lerp_fused.weight", ly["lerp"].reshape(6, 1, 1, S.dim))
        t(p + "time_mix_receptance.weight", ly["rw"]); t(p + "time_mix_key.weight", ly["kw"])
        t(p + "time_mix_value.weight", ly["vw"]); t(p + "time_mix_output.weight", ly["ow"])
        # GGUF keeps the LoRA factors as logical (out,in) of their own product
        for nm, key in (("w1", "w1"), ("w2", "w2"), ("a1", "a1"), ("a2", "a2"),
                        ("v1", "v1"), ("v2", "v2"), ("g1", "g1"), ("g2", "g2")):
            t(p + f"time_mix_{nm}.weight", ly[key])
        for nm, key in (("w0", "w0"), ("a0", "a0"), ("v0", "v0"), ("k_k", "kk"),
                        ("k_a", "ka"), ("r_k", "rk")):
            t(p + f"time_mix_{nm}.weight", ly[key])
        t(p + "time_mix_ln.weight", ly["lnx_w"]); t(p + "time_mix_ln.bias", ly["lnx_b"])
        t(p + "channel_mix_key.weight", ly["cmk"]); t(p + "channel_mix_value.weight", ly["cmv"])
        t(p + "channel_mix_lerp_k.weight", ly["cmk_lerp"])
    t("output_norm.weight", w.on_w)
    t("output_norm.bias", w.on_b)
    t("output.weight", w.head)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()


def make_rwkv(out: Path, ref_root: Path):
    sys.path.insert(0, str(ref_root))
    sys.path.insert(0, str(ref_root / "experiments"))
    from sunnynet.runtime import quant as Q
    from sunnynet.runtime.rwkv7 import RWKV7
    # the reference INT4 exporter loads its quantiser through ctypes; point it at
    # the reference build in oracle/_ref instead of its read-only build folder
    Q.DLL = oracle.REF_ABI_SO
    Q._needs_rebuild = lambda: False
    import _export_rwkv7 as EX

    shape = formats.RWKV_PRESETS["tiny"]
    seed = 3
    w = formats.random_rwkv(shape, seed)
    res = {"shape": np.array([shape.layers, shape.dim, shape.head_size, shape.ffn, shape.vocab,
                              *shape.ranks], np.int32), "seed": np.int32(seed)}
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        gg = td / "m.gguf"
        _write_gguf(gg, w)
        blobs = {}
        for kind, extra in (("fp32", ["--f32"]), ("q4", [])):
            dst = td / f"m.{kind}.bin"
            old = sys.argv
            sys.argv = ["_export_rwkv7.py", str(gg), str(dst)] + extra
            try:
                EX.main()
            finally:
                sys.argv = old
            blobs[kind] = dst
            mine = td / f"mine.{kind}.bin"
            formats.write_krwk(mine, w, quant=kind)
            assert mine.read_bytes() == dst.read_bytes(), f"write_krwk({kind}) differs"
            res[f"sha_{kind}"] = np.array(sha(dst))
        mine4 = td / "mine.q4g.bin"
        formats.write_krwk(mine4, w, quant="q4g", group=128)
        res["sha_q4g"] = np.array(sha(mine4))

        ref = RWKV7(gg)
        rng = np.random.default_rng(9)
        toks = rng.integers(0, shape.vocab, 16).astype(np.int32)
        st = ref.reset(ref.init_state())
        ln = np.stack([ref.step(int(t), st) for t in toks]).astype(np.float32)
        res["tokens"], res["logits_numpy"] = toks, ln
        res["S_numpy"], res["shift_numpy"] = st["S"].copy(), st["shift"].copy()
        RA = oracle.ref_abi()
        for kind, blob in blobs.items():
            h = RA.sn_rk_load(str(blob).encode())
            assert h
            lg = np.empty((16, shape.vocab), np.float32)
            for i, t in enumerate(toks):
                RA.sn_rk_step(h, int(t), P(lg[i]))
            dbg = np.empty(9 * shape.dim, np.float32)
            RA.sn_rk_reset(h)
            RA.sn_rk_dbg(h, int(toks[0]), 1, P(dbg))
            RA.sn_rk_free(h)
            res[f"logits_c_{kind}"] = lg
            res[f"dbg_c_{kind}"] = dbg
    np.savez_compressed(out / "rwkv_tiny.npz", **res)


# ------------------------------------------- the reference's ctypes bindings
def _ctype_name(t) -> str:
    if t is None:
        return "void"
    if getattr(t, "_type_", None) is ctypes.c_float and issubclass(t, ctypes._Pointer):
        return "float_p"
    return {ctypes.c_void_p: "void_p", ctypes.c_char_p: "char_p", ctypes.c_int: "int",
            ctypes.c_uint32: "uint32", ctypes.c_int32: "int", ctypes.c_float: "float",
            ctypes.c_int64: "int64"}[t]


class _Recorder:
    """Stands in for the CDLL a reference loader opens: records every
    restype/argtypes assignment the loader makes."""

    def __init__(self):
        object.__setattr__(self, "fns", {})

    def __getattr__(self, name):
        fns = object.__getattribute__(self, "fns")
        if name not in fns:
            fns[name] = _RecFn()
        return fns[name]


class _RecFn:
    def __init__(self):
        self.restype = ctypes.c_int  # ctypes' default
        self.argtypes = None


def make_ref_bindings(out: Path, ref_root: Path):
    """Every symbol the reference's ctypes loaders bind (runtime/__init__.py
    load_runtime, model.py _load, abi.py load_abi, quant.py load_quant,
    rwkv7_c.py _load, kernels/__init__.py load_kernel) with the argtypes/
    restype they set, and every function the reference's runtime headers
    declare."""
    import importlib
    import json
    import re
    sys.path.insert(0, str(ref_root))
    loaders = {"__init__": "load_runtime", "model": "_load", "abi": "load_abi",
               "quant": "load_quant", "rwkv7_c": "_load", "kernels": "load_kernel"}
    real_cdll = ctypes.CDLL
    res = {"loaders": {}, "headers": {}}
    try:
        for modname, fn in loaders.items():
            full = ("sunnynet.kernels" if modname == "kernels" else
                    "sunnynet.runtime" + ("" if modname == "__init__" else "." + modname))
            mod = importlib.import_module(full)
            rec = _Recorder()
            ctypes.CDLL = lambda *a, **k: rec
            for attr, val in (("_find_gcc", lambda: "gcc"), ("_needs_rebuild", lambda: False),
                              ("_lib", None)):
                if hasattr(mod, attr):
                    setattr(mod, attr, val)
            getattr(mod, fn)()
            where = ("kernels/__init__.py" if modname == "kernels" else
                     f"runtime/{modname}.py")
            res["loaders"][f"{where}:{fn}"] = {
                name: {"restype": _ctype_name(f.restype),
                       "argtypes": [_ctype_name(t) for t in (f.argtypes or [])]}
                for name, f in sorted(object.__getattribute__(rec, "fns").items())}
            if hasattr(mod, "_lib"):
                mod._lib = None
    finally:
        ctypes.CDLL = real_cdll
    for h in ("sn_abi.h", "recur.h", "quant.h", "sunnynet.h", "rwkv7.h"):
        txt = (ref_root / "sunnynet" / "runtime" / h).read_text(encoding="utf-8")
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        txt = re.sub(r"//.*", "", txt)
        txt = re.sub(r"#.*", "", txt)
        names = sorted({m.group(1) for m in re.finditer(r"\b(sn_[A-Za-z0-9_]*)\s*\(", txt)})
        res["headers"][h] = names
    (out / "ref_bindings.json").write_text(json.dumps(res, indent=1, sort_keys=True) + "\n")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference checkout")
    args = ap.parse_args()
    oracle.build(ref_root=args.ref)
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref not built (reference tree missing?)")
    make_prims(HERE)
    make_sunny(HERE, Path(args.ref))
    make_rwkv(HERE, Path(args.ref))
    make_ref_bindings(HERE, Path(args.ref))
    for f in sorted(HERE.glob("*")):
        if f.suffix in (".npz", ".usnn"):
            print(f"{f.name}: {f.stat().st_size} bytes")


if __name__ == "__main__":
    main()
