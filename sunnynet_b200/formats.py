"""Weight blob formats and seeded synthetic models.

Formats (all little-endian):

* **USNN** -- the reference's fp32 SunnyNet blob (``release.py:93-141``): a
  ``<10i`` header ``{0x4E4E5355, vocab, dim, inner, rank, taps, layers, group=8,
  tied=1, clamp}``, then per layer ``ni_g[D] ni_c[D] nm_g[I] nm_c[I] dw(K,D)
  Vt(D,R) Ut(R,2D) Wzt(D,I) Wct(I,D) Wst(D,D) delta[D] {tanh(a), b_gain}``, then
  ``eps p_floor no_g[D] no_c[D] embed(V,D) headt(D,V)``. Matrices are stored
  transposed, (in,out). ``Ws`` is ``W_s`` with the circulant filter folded in.
* **USNQ** -- this project's INT8 SunnyNet blob (the reference has none,
  ``release.py:8-10``): a ``<12i`` header ``{0x514E5355, version=1, vocab, dim,
  inner, rank, taps, layers, group, tied, clamp, qbits=8}``, the same small
  tensors as USNN, and each GEMV matrix (and the LM head) as (out,in) row-major
  int8 codes followed by one fp32 scale per output row, produced by the
  reference's symmetric INT8 quantiser with ``block = in`` (``recur.c:134-161``).
  The embedding stays fp32 (it is a lookup, not a GEMV).
* **KRWK v3** -- the reference's RWKV-7 blob (``experiments/_export_rwkv7.py``):
  ``<10i`` header ``{0x4B57524B, 3, L, D, HS, NH, F, g_rank, vocab, q4}``, eps,
  ``L x <4i`` LoRA ranks, then a tagged tensor stream (tag 0: fp32 (in,out);
  tag 1: INT4 (out,in/2) codes + (out,in/64) fp32 scales).
* **KRWK v4** -- this project's RWKV-7 blob with INT4 group G and fp16 scales
  (the reference's loader rejects unknown versions, ``rwkv7.c:419-422``): the
  v3 layout with version 4, an extra int32 ``group`` after eps, and tag 2 for
  INT4 (out,in/2) codes + (out,in/G) fp16 scales. fp16 scale = fp16(amax/7);
  codes are computed against the stored fp16 value.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

USNN_MAGIC = 0x4E4E5355
USNQ_MAGIC = 0x514E5355
KRWK_MAGIC = 0x4B57524B

F32 = np.float32


# ----------------------------------------------------------------- quantisers
def quant_i8_rows(x: np.ndarray):
    """Symmetric INT8, one block per row (recur.c:134-161 with block = N)."""
    x = np.ascontiguousarray(x, F32)
    amax = np.abs(x).max(axis=1)
    sc = np.where(amax > 0, amax / F32(127.0), F32(1.0)).astype(F32)
    inv = (F32(1.0) / sc).astype(F32)
    q = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    return q, sc


def quant_i4(w: np.ndarray, block: int, fp16_scale: bool = False):
    """Group-symmetric INT4 of an (out,in) matrix (quant.c:34-65).

    Returns codes (out, in/2) uint8 -- byte k of a group holds value k in the low
    nibble and value k+block/2 in the high nibble -- and scales (out, in/block)
    as fp32 or, with ``fp16_scale``, fp16(amax/7) (codes against that value).
    """
    w = np.ascontiguousarray(w, F32)
    out, n = w.shape
    assert n % block == 0 and block % 2 == 0
    g = w.reshape(out, n // block, block)
    amax = np.abs(g).max(axis=2)
    sc = np.where(amax > 0, amax / F32(7.0), F32(1.0)).astype(F32)
    if fp16_scale:
        sc16 = sc.astype(np.float16)
        sc16 = np.where(sc16 == 0, np.float16(np.finfo(np.float16).smallest_subnormal), sc16)
        sc = sc16.astype(F32)
    inv = (F32(1.0) / sc).astype(F32)
    v = np.clip(np.rint(g * inv[:, :, None]), -8, 7).astype(np.int32) + 8
    half = block // 2
    codes = (v[:, :, :half] | (v[:, :, half:] << 4)).astype(np.uint8).reshape(out, n // 2)
    return codes, (sc16 if fp16_scale else sc)


def dequant_i4(codes: np.ndarray, sc: np.ndarray, block: int) -> np.ndarray:
    out = codes.shape[0]
    n = codes.shape[1] * 2
    c = codes.reshape(out, n // block, block // 2).astype(np.int32)
    v = np.concatenate([(c & 0x0F) - 8, (c >> 4) - 8], axis=2).astype(F32)
    return (v * sc.astype(F32)[:, :, None]).reshape(out, n)


# ------------------------------------------------------------------ SunnyNet
@dataclass
class SunnyShape:
    vocab: int
    dim: int
    inner: int
    rank: int
    taps: int = 4
    layers: int = 4
    group: int = 8
    h_min: float = 2.0
    h_max: float = 8192.0

    @property
    def kh(self) -> int:
        return max(self.taps - 1, 1)


# inner/rank follow the reference's own preset ratio (SunnyConfig.proto20m,
# model.py:45-47: d512 -> i896 r320).
SUNNY_PRESETS = {
    "c2": SunnyShape(16384, 512, 896, 320, 4, 4),
    "c3": SunnyShape(32000, 768, 1344, 480, 4, 12),
    "c5": SunnyShape(32000, 1536, 2688, 960, 4, 24),
    "tiny": SunnyShape(512, 64, 96, 32, 4, 2),
}


@dataclass
class SunnyWeights:
    """Model-layout weights: matrices are (out,in), y = W x."""
    shape: SunnyShape
    layers: list = field(default_factory=list)
    no_g: np.ndarray | None = None
    no_c: np.ndarray | None = None
    embed: np.ndarray | None = None
    head: np.ndarray | None = None   # (vocab, D); None = tied to embed (the reference's only mode)
    eps: float = 0.02 * 0.02 + 1e-5  # CenteredScaleNorm s_min^2 + eps (ops.py:38-47)
    clamp: int = 0


def _orth(rng: np.random.Generator, out_f: int, in_f: int, rho: float) -> np.ndarray:
    """Orthogonal slice with spectral radius rho (init.py:9-22 semantics)."""
    n = max(out_f, in_f)
    a = rng.standard_normal((n, n), dtype=np.float32)
    q, r = np.linalg.qr(a)
    d = np.sign(np.diagonal(r))
    d[d == 0] = 1
    q = q * d[None, :]
    return np.ascontiguousarray(q[:out_f, :in_f] * rho, F32)


def random_sunny(shape: SunnyShape, seed: int = 0, perturb: bool = False,
                 fast: bool = False) -> SunnyWeights:
    """Seeded random-init SunnyNet with the reference's init distributions.

    Embedding N(0, 0.02) (model.py:72); V, U, W_z, W_c orthogonal with rho=1 and
    W_s with rho=0.5 (layers.py:150-157); depthwise taps N(0,1)*0.1; circulant
    taps (0.25, 0.5, 0.25); a = b_gain = 0.5; horizons log-spaced over
    [h_min, h_max] through theta = logit((i+0.5)/D) (ops.py:61-64, layers.py:137).
    ``perturb`` moves the norm gains/centres and a/b_gain off their init values
    so parity tests exercise every parameter. ``fast`` replaces the QR-based
    orthogonal draws by scaled Gaussians (same scale, for large timing runs).
    """
    S = shape
    rng = np.random.default_rng(seed)
    D, I, R, K = S.dim, S.inner, S.rank, S.taps

    def mat(o, i, rho):
        if fast:
            return (rng.standard_normal((o, i), dtype=np.float32) *
                    F32(rho / math.sqrt(max(o, i)))).astype(F32)
        return _orth(rng, o, i, rho)

    w = SunnyWeights(shape=S)
    th = (np.arange(D, dtype=np.float64) + 0.5) / D
    theta = np.log(th) - np.log1p(-th)
    span = math.log(S.h_max / S.h_min)
    H = S.h_min * np.exp(span / (1.0 + np.exp(-theta)))
    delta = (1.0 / H).astype(F32)
    for _ in range(S.layers):
        ly = {
            "ni_g": np.ones(D, F32), "ni_c": np.zeros(D, F32),
            "nm_g": np.ones(I, F32), "nm_c": np.zeros(I, F32),
            "dw": (rng.standard_normal((D, K), dtype=np.float32) * F32(0.1)).astype(F32),
            "V": mat(R, D, 1.0), "U": mat(2 * D, R, 1.0),
            "Wz": mat(I, D, 1.0), "Wc": mat(D, I, 1.0),
        }
        Ws = mat(D, D, 0.5)
        t0, t1, t2 = F32(0.25), F32(0.5), F32(0.25)
        ly["Ws_eff"] = ((t0 * np.roll(Ws, -1, axis=1) + t1 * Ws) + t2 * np.roll(Ws, 1, axis=1)).astype(F32)
        ly["delta"] = delta.copy()
        a, b = 0.5, 0.5
        if perturb:
            for k, n in (("ni_g", D), ("nm_g", I)):
                ly[k] = (1.0 + 0.1 * rng.standard_normal(n)).astype(F32)
            for k, n in (("ni_c", D), ("nm_c", I)):
                ly[k] = (0.05 * rng.standard_normal(n)).astype(F32)
            a, b = 0.5 + 0.3 * rng.standard_normal(), 0.5 + 0.2 * rng.standard_normal()
        ly["a_tanh"] = float(np.float32(math.tanh(a)))
        ly["b_gain"] = float(np.float32(b))
        w.layers.append(ly)
    w.no_g = np.ones(D, F32)
    w.no_c = np.zeros(D, F32)
    if perturb:
        w.no_g = (1.0 + 0.1 * rng.standard_normal(D)).astype(F32)
        w.no_c = (0.05 * rng.standard_normal(D)).astype(F32)
    w.embed = (rng.standard_normal((S.vocab, D), dtype=np.float32) * F32(0.02)).astype(F32)
    return w


_MATS = ("V", "U", "Wz", "Wc", "Ws_eff")


def write_usnn(path, w: SunnyWeights) -> int:
    """Write the reference fp32 USNN blob (byte-compatible with release.py)."""
    S = w.shape
    parts = [struct.pack("<10i", USNN_MAGIC, S.vocab, S.dim, S.inner, S.rank, S.taps,
                         S.layers, S.group, 1, int(w.clamp))]
    put = lambda a: parts.append(np.ascontiguousarray(a, F32).tobytes())
    for ly in w.layers:
        put(ly["ni_g"]); put(ly["ni_c"]); put(ly["nm_g"]); put(ly["nm_c"])
        put(ly["dw"].T)
        for k in _MATS:
            put(ly[k].T)
        put(ly["delta"])
        parts.append(struct.pack("<2f", ly["a_tanh"], ly["b_gain"]))
    parts.append(struct.pack("<2f", w.eps, 1.0 / S.h_max))
    put(w.no_g); put(w.no_c); put(w.embed)
    put((w.embed if w.head is None else w.head).T)
    buf = b"".join(parts)
    Path(path).write_bytes(buf)
    return len(buf)


def write_usnq(path, w: SunnyWeights) -> int:
    """Write the INT8 per-output-row USNQ blob (see module docstring)."""
    S = w.shape
    parts = [struct.pack("<12i", USNQ_MAGIC, 1, S.vocab, S.dim, S.inner, S.rank, S.taps,
                         S.layers, S.group, 1, int(w.clamp), 8)]
    put = lambda a: parts.append(np.ascontiguousarray(a, F32).tobytes())

    def putq(m):
        q, sc = quant_i8_rows(m)
        parts.append(q.tobytes())
        parts.append(sc.tobytes())

    for ly in w.layers:
        put(ly["ni_g"]); put(ly["ni_c"]); put(ly["nm_g"]); put(ly["nm_c"])
        put(ly["dw"].T)
        for k in _MATS:
            putq(ly[k])
        put(ly["delta"])
        parts.append(struct.pack("<2f", ly["a_tanh"], ly["b_gain"]))
    parts.append(struct.pack("<2f", w.eps, 1.0 / S.h_max))
    put(w.no_g); put(w.no_c); put(w.embed)
    putq(w.embed if w.head is None else w.head)
    buf = b"".join(parts)
    Path(path).write_bytes(buf)
    return len(buf)


def read_sunny_header(path) -> dict:
    with open(path, "rb") as f:
        h = struct.unpack("<10i", f.read(40))
        if h[0] == USNN_MAGIC:
            return dict(kind="usnn", vocab=h[1], dim=h[2], inner=h[3], rank=h[4], taps=h[5],
                        layers=h[6], group=h[7], tied=h[8], clamp=h[9])
        if h[0] == USNQ_MAGIC:
            h2 = struct.unpack("<2i", f.read(8))
            return dict(kind="usnq", version=h[1], vocab=h[2], dim=h[3], inner=h[4], rank=h[5],
                        taps=h[6], layers=h[7], group=h[8], tied=h[9], clamp=h2[0], qbits=h2[1])
    raise ValueError(f"{path}: not a SunnyNet blob")


# --------------------------------------------------------------------- RWKV-7
@dataclass
class RwkvShape:
    layers: int = 12
    dim: int = 768
    head_size: int = 64
    ffn: int = 3072
    vocab: int = 65536
    ranks: tuple = (64, 64, 32, 128)  # (w, a, v, g) LoRA ranks

    @property
    def n_head(self) -> int:
        return self.dim // self.head_size


RWKV_PRESETS = {
    "c4": RwkvShape(12, 768, 64, 3072, 65536, (64, 64, 32, 128)),
    "tiny": RwkvShape(2, 128, 64, 512, 512, (32, 32, 16, 64)),
}

# Matrices in stream order per layer: name -> (out_dim key, in_dim key)
_RK_MATS = ("rw", "kw", "vw", "ow", "w1", "w2", "a1", "a2", "v1", "v2", "g1", "g2")


@dataclass
class RwkvWeights:
    """Logical weights: matrices are (out,in), y = W x."""
    shape: RwkvShape
    layers: list = field(default_factory=list)
    en_w: np.ndarray | None = None
    en_b: np.ndarray | None = None
    on_w: np.ndarray | None = None
    on_b: np.ndarray | None = None
    embed: np.ndarray | None = None
    head: np.ndarray | None = None  # (vocab, D)
    eps: float = 1e-5


def random_rwkv(shape: RwkvShape, seed: int = 0) -> RwkvWeights:
    """Seeded random-init RWKV-7: matrices N(0, fan_in^-1/2), norm gains 1+N(0,0.1),
    lerps 0.5+N(0,0.2), w0/a0/v0/k_k/k_a/r_k N(0,0.3)."""
    S = shape
    rng = np.random.default_rng(seed)
    D, F = S.dim, S.ffn
    Rw, Ra, Rv, Rg = S.ranks

    def m(o, i):
        return (rng.standard_normal((o, i), dtype=np.float32) * F32(1.0 / math.sqrt(i))).astype(F32)

    def v(n, mu, sd):
        return (mu + sd * rng.standard_normal(n)).astype(F32)

    w = RwkvWeights(shape=S)
    for _ in range(S.layers):
        ly = {
            "ln1w": v(D, 1, 0.1), "ln1b": v(D, 0, 0.1), "ln2w": v(D, 1, 0.1), "ln2b": v(D, 0, 0.1),
            "lerp": v(6 * D, 0.5, 0.2).reshape(6, D),
            "rw": m(D, D), "kw": m(D, D), "vw": m(D, D), "ow": m(D, D),
            "w1": m(Rw, D), "w2": m(D, Rw), "a1": m(Ra, D), "a2": m(D, Ra),
            "v1": m(Rv, D), "v2": m(D, Rv), "g1": m(Rg, D), "g2": m(D, Rg),
            "w0": v(D, 0, 0.3), "a0": v(D, 0, 0.3), "v0": v(D, 0, 0.3),
            "kk": v(D, 0, 0.3), "ka": v(D, 0, 0.3), "rk": v(D, 0, 0.3),
            "lnx_w": v(D, 1, 0.1), "lnx_b": v(D, 0, 0.1),
            "cmk": m(F, D), "cmv": m(D, F), "cmk_lerp": v(D, 0.5, 0.2),
        }
        w.layers.append(ly)
    w.en_w, w.en_b = v(D, 1, 0.1), v(D, 0, 0.1)
    w.on_w, w.on_b = v(D, 1, 0.1), v(D, 0, 0.1)
    w.embed = (rng.standard_normal((S.vocab, D), dtype=np.float32) * F32(0.5)).astype(F32)
    w.head = m(S.vocab, D)
    return w


def write_krwk(path, w: RwkvWeights, quant: str = "fp32", group: int = 128) -> dict:
    """Write a KRWK blob. quant: "fp32" (v3, all fp32), "q4" (v3, INT4 block 64
    fp32 scales, as the reference exporter), or "q4g" (v4, INT4 group `group`
    fp16 scales). Matrices whose in-dim is not a multiple of the block stay fp32
    (_export_rwkv7.py:192-193)."""
    S = w.shape
    D, HS, NH, F = S.dim, S.head_size, S.n_head, S.ffn
    version = 4 if quant == "q4g" else 3
    block = group if quant == "q4g" else 64
    parts = [struct.pack("<10i", KRWK_MAGIC, version, S.layers, D, HS, NH, F,
                         S.ranks[3], S.vocab, 0 if quant == "fp32" else 1),
             struct.pack("<f", w.eps)]
    if version == 4:
        parts.append(struct.pack("<i", group))
    for _ in range(S.layers):
        parts.append(struct.pack("<4i", *S.ranks))
    stats = {"int4_mats": 0, "f32_mats": 0}

    def put(a):
        parts.append(struct.pack("<i", 0))
        parts.append(np.ascontiguousarray(a, F32).reshape(-1).tobytes())

    def putm(W):  # W logical (out,in)
        out_d, in_d = W.shape
        if quant != "fp32" and in_d % block == 0 and out_d > 0:
            codes, sc = quant_i4(W, block, fp16_scale=(quant == "q4g"))
            parts.append(struct.pack("<i", 2 if quant == "q4g" else 1))
            parts.append(codes.tobytes() + sc.tobytes())
            stats["int4_mats"] += 1
        else:
            parts.append(struct.pack("<i", 0))
            parts.append(np.ascontiguousarray(W.T, F32).tobytes())
            stats["f32_mats"] += 1

    for ly in w.layers:
        put(ly["ln1w"]); put(ly["ln1b"]); put(ly["ln2w"]); put(ly["ln2b"]); put(ly["lerp"])
        for k in _RK_MATS:
            putm(ly[k])
        for k in ("w0", "a0", "v0", "kk", "ka", "rk", "lnx_w", "lnx_b"):
            put(ly[k])
        putm(ly["cmk"]); putm(ly["cmv"]); put(ly["cmk_lerp"])
    put(w.en_w); put(w.en_b); put(w.on_w); put(w.on_b); put(w.embed)
    putm(w.head)
    buf = b"".join(parts)
    Path(path).write_bytes(buf)
    return {"bytes": len(buf), **stats}
