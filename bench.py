"""Benchmark of the SunnyNet token loop on B200s (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]

Workloads (synthetic seeded inputs, random-init weights):
  c1   gated scan, B=1 T=4096 C=1024 (one step = one full scan)
  c2   SunnyNet small decode (L4 d512 i896 r320 V16384, fp32), B=256 per GPU
  c2b1 the same model at B=1
  c3   (default) SunnyNet 100M-class (L12 d768 i1344 r480 V32000), INT8
       per-row weights, a global batch of 1024 split over the GPUs
       (1024/512/256/128 per GPU at 1/2/4/8: strong scaling), after a
       2048-token chunked prefill. On one GPU the line also carries the
       metric's other batch sizes as sub-records: c2 at B=256 and at B=1.
  c4   RWKV-7 191M shape, INT4 group-128 fp16 scales, B=64 per GPU (c4b1, c4b512)
  c5   chunked prefill, SunnyNet 0.5B shape (L24 d1536 i2688 r960 V32000) fp32,
       T=32768 in chunks of 256, 8 sequences per GPU

A step is one pass of the hot path over one batch: one decode token for every
sequence of the batch (or one full scan for c1, one 256-token chunk for c5).
Sequences are independent and shard by batch over the ranks (no collective on
the data path); timing is the max over ranks of CUDA-event time.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


# ------------------------------------------------------------------ helpers
def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "src": "fallback"}


def profile_traffic(kernel_key: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    for f in sorted((REPO / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            m = re.match(r"traffic_bytes_per_launch\[(.+?)\]:\s*([0-9.eE+]+)", line.strip())
            if m and m.group(1) == kernel_key:
                return float(m.group(2))
    return None


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while running."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def shard(total: int, world: int, rank: int):
    """Sequences [start, start + count) that `rank` owns when `total`
    independent sequences are split over `world` ranks: contiguous ranges whose
    sizes differ by at most one, covering every sequence exactly once."""
    base, extra = divmod(total, world)
    count = base + (1 if rank < extra else 0)
    return rank * base + min(rank, extra), count


class Dist:
    """One process per GPU (torchrun's RANK / LOCAL_RANK / WORLD_SIZE). The
    data path has no collective (sequences are independent); the process
    group only lines the ranks up around the timed region and takes the max
    of their times. backend="gloo", cuda=False runs the same logic on CPU."""

    def __init__(self, backend: str = "nccl", cuda: bool = True):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend, self.cuda = backend, cuda
        self.pg = None

    def init(self, torch):
        if self.cuda:
            torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            kw = {"device_id": torch.device("cuda", self.local)} if self.cuda else {}
            dist.init_process_group(self.backend, timeout=datetime.timedelta(seconds=120), **kw)
            self.pg = dist

    def barrier(self, torch):
        if self.cuda:
            torch.cuda.synchronize()
        if self.pg:
            self.pg.barrier()
        if self.cuda:
            torch.cuda.synchronize()

    def max(self, torch, v: float) -> float:
        if not self.pg:
            return v
        t = torch.tensor([v], device="cuda" if self.cuda else "cpu", dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def gather(self, torch, values) -> list:
        """Every rank's equal-length list of numbers, in rank order (host-side
        collection of per-rank results such as token counts or checksums)."""
        t = torch.tensor(list(values), device="cuda" if self.cuda else "cpu",
                         dtype=torch.float64)
        if not self.pg:
            return [t.tolist()]
        out = [torch.empty_like(t) for _ in range(self.world)]
        self.pg.all_gather(out, t)
        return [o.tolist() for o in out]

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def timed_steps(torch, dist, step, K: int, W: int, flush=None):
    """W warm-up steps, then K timed steps bracketed by barrier+sync; each step
    is bracketed by CUDA events on the current stream, with an untimed L2
    flush before it when `flush` is given. Returns (ms per step, max over ranks)."""
    for _ in range(W):
        if flush is not None:
            flush()
        step()
    dist.barrier(torch)
    st = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(K)]
    for s, e in evs:
        if flush is not None:
            flush()
        s.record(st)
        step()
        e.record(st)
    dist.barrier(torch)
    ms = sum(s.elapsed_time(e) for s, e in evs) / K
    return dist.max(torch, ms)


def keep_busy(torch, step, seconds: float = 1.5, inner: int = 20):
    """Run the same step for `seconds` more (untimed) so the clock sampler,
    which polls every 200 ms, sees the GPU under this load even when the K
    timed steps take only a few milliseconds."""
    t_end = time.time() + seconds
    while time.time() < t_end:
        for _ in range(inner):
            step()
        torch.cuda.synchronize()


# ---------------------------------------------------------------- workloads
def wl_c1(args, torch, dist, ours: bool):
    """Gated scan, BASELINE config 1. One step = one scan of B*T*C elements.

    Headline: scan mode 1 (chunked in T, three kernels), within 1e-4 of the
    reference. Mode 0 (sequential per channel, bit-exact) is timed beside it."""
    B, T, N = 1, 4096, 1024
    rng = np.random.default_rng(0)
    H = np.exp(np.linspace(np.log(2.0), np.log(8192.0), N))
    a = rng.uniform(1.0 - 1.0 / H, 1.0, (B, T, N)).astype(np.float32)
    u = rng.standard_normal((B, T, N)).astype(np.float32)
    s0 = np.zeros((B, N), np.float32)
    alg_bytes = 3 * B * T * N * 4  # read a, u; write out (+ B*N*8 for s0/send, negligible)
    res = {"metric": "gated scan throughput (algorithmic bytes)", "unit": "GB/s",
           "higher_is_better": True, "dtype": "f32",
           "config": {"workload": "c1 gated scan B=1 T=4096 C=1024", "l2": "flushed between steps",
                      "inputs": "a~U[1-1/H,1], H log-spaced [2,8192]; u~N(0,1); s0=0; seed 0",
                      "scan_mode": "1 (chunked; outputs within 1e-4 of the reference)"}}
    if not ours:
        return res, ref_scan(a, u, s0, alg_bytes)
    from sunnynet_b200 import runtime, _lib
    lib = runtime.load_runtime()
    from sunnynet_b200._lib import check, ptr
    da, du, ds = (torch.from_numpy(x).cuda() for x in (a, u, s0))
    out = torch.empty_like(da)
    send = torch.empty_like(ds)
    check(lib.sn_abi_cuda_set_stream(torch.cuda.current_stream().cuda_stream))
    check(lib.sn_abi_cuda_set_async(1))
    flushbuf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    peaks = measured_peaks()

    def step():
        check(lib.sn_abi_recur_scan(ptr(da), ptr(du), ptr(ds), ptr(out), ptr(send), B, T, N, 1))

    old_mode = lib.sn_abi_cuda_scan_mode(0)
    ms_exact = timed_steps(torch, dist, step, args.steps, args.warmup, flush=flushbuf.zero_)
    lib.sn_abi_cuda_scan_mode(1)
    with ClockSampler(dist.local) as clk:
        ms = timed_steps(torch, dist, step, args.steps, args.warmup, flush=flushbuf.zero_)
        keep_busy(torch, step, inner=200)
    # per-kernel device time of the mode-1 scan (CUDA events around each kernel)
    check(lib.sn_abi_cuda_profile(1))
    for _ in range(5):
        flushbuf.zero_()
        step()
    torch.cuda.synchronize()
    check(lib.sn_abi_cuda_profile(0))
    fams = _lib.profile_report()
    check(lib.sn_abi_cuda_set_async(0))
    # end-to-end: the public call with pinned host buffers (H2D + kernels + D2H)
    pa = torch.from_numpy(a).pin_memory()
    pu = torch.from_numpy(u).pin_memory()
    ps = torch.from_numpy(s0).pin_memory()
    po = torch.empty_like(pa).pin_memory()
    pe = torch.empty_like(ps).pin_memory()
    for _ in range(3):
        check(lib.sn_abi_recur_scan(ptr(pa), ptr(pu), ptr(ps), ptr(po), ptr(pe), B, T, N, 1))
    reps = 20
    t0 = time.perf_counter()
    for _ in range(reps):
        check(lib.sn_abi_recur_scan(ptr(pa), ptr(pu), ptr(ps), ptr(po), ptr(pe), B, T, N, 1))
    e2e_s = (time.perf_counter() - t0) / reps
    e2e_s = dist.max(torch, e2e_s)
    lib.sn_abi_cuda_scan_mode(old_mode)
    achieved = alg_bytes / (ms * 1e-3) / 1e9
    ach_exact = alg_bytes / (ms_exact * 1e-3) / 1e9
    kern = {k: {"launches": n, "avg_us": t / n * 1e3} for k, (n, t) in fams.items()}
    tot = sum(v["avg_us"] for v in kern.values()) or 1.0
    for v in kern.values():
        v["share"] = v["avg_us"] / tot
    res.update({
        "ms_per_step": ms,
        "value": achieved * dist.world,
        "e2e": {"value": alg_bytes * dist.world / e2e_s / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": int(2 * B * T * N * 4 + B * N * 4),
                "d2h_bytes_per_step": int(B * T * N * 4 + B * N * 4)},
        # one cooperative launch per step, or agg + carry + apply
        "gpu_launches": (1 if "scan_onepass" in kern else 3) * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "peak_src": peaks["src"],
                     "kernel": "+".join(kern) + " (one mode-1 scan)",
                     "alg_bytes_per_launch": alg_bytes, "kernels": kern,
                     "traffic": profile_traffic("scan_onepass/c1" if "scan_onepass" in kern
                                                else "scan_chunked/c1")},
        "exact_mode": {"ms_per_step": ms_exact, "value": ach_exact * dist.world,
                       "kernel": "scan_exact_kernel", "frac": ach_exact / peaks["hbm_gbs"],
                       "traffic": profile_traffic("scan_exact_kernel/c1")},
        "clocks": clk.summary(),
    })
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = ref_scan(a, u, s0, alg_bytes)
    return res, None


def ref_scan(a, u, s0, alg_bytes, budget_s=3.0):
    """The reference AVX2 sn_recur_scan (oracle/_ref) on the host cores."""
    import oracle
    B, T, N = a.shape
    out = np.empty_like(a)
    se = np.empty((B, N), np.float32)
    P = oracle.ptr
    if oracle.ref_available():
        L, kind = oracle.ref_abi(), "reference"
        fn = lambda: L.sn_recur_scan(P(a), P(u), P(s0), P(out), P(se), B, T, N, 1)
    else:
        L, kind = oracle.lib(), "port"
        fn = lambda: L.or_recur_scan(P(a), P(u), P(s0), P(out), P(se), B, T, N, 1)
    fn()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        fn()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": alg_bytes / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": kind,
            "sample": f"{n} full C1 scans (B=1 T=4096 C=1024); the reference parallelises "
                      f"over B only (recur.c:16), so B=1 runs on one thread"}


def sunny_step_cost(S, B, wbytes, with_head=True):
    """Algorithmic bytes and FLOPs of one decode step for B sequences (weights
    read once, state s + 3-row history ring read, s + newest history row
    written, embedding rows read, logits written)."""
    D, I, R, V, L = S.dim, S.inner, S.rank, S.vocab, S.layers
    mats = D * R + R * 2 * D + D * I + I * D + D * D
    wts = L * mats * wbytes + (V * D * wbytes if with_head else 0)
    if wbytes == 1:  # per-row fp32 scales
        wts += 4 * (L * (R + 2 * D + I + D + D) + (V if with_head else 0))
    state = B * L * (4 * D + 2 * D) * 4
    io = B * D * 4 + (B * V * 4 if with_head else 0)
    flops = 2 * B * (L * mats + (V * D if with_head else 0))
    return wts + state + io, flops


# Families the SunnyNet batched step runs on its side stream (the feedback
# contractions of all layers and the one state split before them), beside
# the layer chain: in the timed graph they overlap the chain's kernels.
SIDE_STREAM = ("gemm_Ws", "split_state")


def family_table(fams, reps: int, ms: float, overlapped=()):
    """Per kernel family of one step: launches, serialised ms (CUDA events
    around each family with the step run kernel by kernel), and that time
    scaled so the chain's families add up to the timed step (`ms`, the graph
    with its overlaps); share = scaled ms / ms. Families in `overlapped` run
    on a side stream beside the chain: scaled by the same factor but marked
    "overlapped" and left out of the sum and of the shares. The fused step's
    per-phase device timestamps ("fused:*") are reported apart: they subdivide
    its one kernel."""
    base = {k: v for k, v in fams.items() if not k.startswith("fused:")}
    tot = sum(v[1] for k, v in base.items() if k not in overlapped) / reps
    scale = ms / tot if tot > 0 else 1.0
    tab = {}
    for k, v in base.items():
        row = {"launches": v[0] / reps, "serial_ms": v[1] / reps, "ms": v[1] / reps * scale}
        if k in overlapped:
            row["overlapped"] = True
        else:
            row["share"] = v[1] / reps * scale / ms
        tab[k] = row
    parts = {k: v[1] / reps for k, v in fams.items() if k.startswith("fused:")}
    return tab, scale, parts


def family_cost(S, B, fam, wbytes):
    """(bytes, flops) per launch of one kernel family of the SunnyNet step."""
    D, I, R, V = S.dim, S.inner, S.rank, S.vocab
    shapes = {"gemm_head": (V, D), "gemm_Wz": (I, D), "gemm_Wc": (D, I), "gemm_Ws": (D, D),
              "gemm_V": (R, D), "gemm_U": (2 * D, R)}
    if fam in shapes:
        n, k = shapes[fam]
        return n * k * wbytes + B * k * 4 + B * n * 4, 2 * B * n * k
    if fam == "fused_step":  # the whole step in one kernel (B <= 8)
        return sunny_step_cost(S, B, wbytes, with_head=True)
    return None, None


def wl_sunny(args, torch, dist, ours, preset, B_total, quant, prefill_T, split):
    from sunnynet_b200 import formats
    S = formats.SUNNY_PRESETS[preset]
    if args.prefill_tokens is not None:
        prefill_T = args.prefill_tokens
    B = shard(B_total, dist.world, dist.rank)[1] if split else B_total
    seqs = B_total if split else B * dist.world  # sequences all ranks step together
    wbytes = 1 if quant else 4
    step_bytes, step_flops = sunny_step_cost(S, B, wbytes)
    res = {"metric": "decode tokens/s", "unit": "tokens/s", "higher_is_better": True,
           "dtype": (("i8w-f32 (INT8 weights exact in bf16; fp32 activations as bf16 hi+lo, "
                      "2 tcgen05 MMAs, fp32 accumulate)" if quant else
                      "f32 (bf16x3 tcgen05 split: hi*hi + hi*lo + lo*hi, fp32 accumulate)")
                     if B >= 16 else ("i8w-f32 (INT8 weights, fp32 FMA)" if quant
                                      else "f32 (fp32 FMA)")),
           "config": {"workload": f"{preset} SunnyNet decode L{S.layers} d{S.dim} i{S.inner} "
                                  f"r{S.rank} V{S.vocab} {'INT8 per-row' if quant else 'fp32'}",
                      "batch_per_gpu": B, "global_batch": seqs,
                      "prefill_tokens": prefill_T, "decode": "greedy, teacher-free",
                      "l2": "flushed between steps" if step_bytes < 2 * (126 << 20) else
                            "working set > L2"}}
    td = tempfile.mkdtemp(prefix="snbench_")
    path = Path(td) / ("m.usnq" if quant else "m.usnn")
    w = formats.random_sunny(S, seed=0)
    (formats.write_usnq if quant else formats.write_usnn)(path, w)
    if not ours:
        ref_path = Path(td) / "ref.usnn"
        if quant:  # the reference has no INT8 SunnyNet: W8A32 = dequantised weights, fp32 blob
            w = dequantised_weights(w)
        formats.write_usnn(ref_path, w)
        return res, ref_sunny(ref_path, S, B_total)
    from sunnynet_b200 import _lib
    from sunnynet_b200._lib import check
    from sunnynet_b200.model import SunnyBatch
    lib = _lib.load()
    check(lib.sn_abi_cuda_set_stream(torch.cuda.current_stream().cuda_stream))
    m = SunnyBatch(path, B)
    g = torch.Generator(device="cuda").manual_seed(dist.rank)
    logits = torch.empty(B, S.vocab, device="cuda")
    check(lib.sn_abi_cuda_set_async(1))
    prompt = torch.randint(0, S.vocab, (B, prefill_T), generator=g, device="cuda",
                           dtype=torch.int32)
    if prefill_T >= 256:  # the chunked prefill path (256-token chunks, state carried)
        m.prefill(prompt, chunk=256, logits=logits)
    else:
        for t in range(prefill_T):
            m.step(prompt[:, t].contiguous(), logits=logits)
    cur = torch.argmax(logits, dim=1).to(torch.int32).contiguous()

    def step():
        m.step_argmax(cur, out=cur)

    flushbuf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    flush = flushbuf.zero_ if step_bytes < 2 * (126 << 20) else None
    with ClockSampler(dist.local) as clk:
        ms = timed_steps(torch, dist, step, args.steps, args.warmup, flush=flush)
        if args.ncu:
            res.update({"ms_per_step": ms, "value": seqs / (ms * 1e-3),
                        "note": "--ncu run: launch list only, no other measurements"})
            m.close()
            return res, None
        keep_busy(torch, step)
    # host-side collection of every rank's greedy tokens (a checksum per rank)
    toks = cur.to(torch.int64)
    res["tokens_per_rank"] = [int(v[0]) for v in dist.gather(torch, [int(toks.numel())])]
    res["token_checksums"] = [int(v[0]) for v in dist.gather(torch, [int(toks.sum().item())])]
    # live per-kernel timing: CUDA events around every kernel family of the
    # same step run without its graph (serialised); scaled to the timed step
    # below so the families' shares add up to it
    check(lib.sn_abi_cuda_profile(1))
    for _ in range(3):
        if flush:
            flush()
        step()
    torch.cuda.synchronize()
    check(lib.sn_abi_cuda_profile(0))
    fams = _lib.profile_report()
    check(lib.sn_abi_cuda_set_async(0))
    tab, scale, parts = family_table(fams, 3, ms, SIDE_STREAM)
    # the dominant kernel: the family of the layer chain with a work model
    # taking the most step time
    known = [k for k in tab
             if family_cost(S, B, k, wbytes)[0] is not None and not tab[k].get("overlapped")]
    dom = max(known, key=lambda k: tab[k]["ms"])
    n_l = tab[dom]["launches"]
    fb, ff = family_cost(S, B, dom, wbytes)
    peaks = measured_peaks()
    per_launch_s = tab[dom]["ms"] / n_l * 1e-3
    if B >= 64 and ff:
        rl = {"bound": "tensor", "achieved": ff / per_launch_s / 1e12,
              "peak": peaks["bf16_tflops"], "unit": "TFLOP/s"}
    else:
        rl = {"bound": "hbm", "achieved": (fb or 0) / per_launch_s / 1e9,
              "peak": peaks["hbm_gbs"], "unit": "GB/s"}
    rl.update({"frac": rl["achieved"] / rl["peak"], "peak_src": peaks["src"], "kernel": dom,
               "launches": n_l, "avg_launch_us": per_launch_s * 1e6,
               "avg_launch_us_serialised": tab[dom]["serial_ms"] / n_l * 1e3,
               "alg_bytes_per_launch": fb, "alg_flops_per_launch": ff,
               "traffic": profile_traffic(f"{dom}/{preset}/B{B}"),
               "step_alg_bytes": step_bytes, "step_alg_flops": step_flops,
               "step_hbm_gbs": step_bytes / (ms * 1e-3) / 1e9,
               "step_tflops": step_flops / (ms * 1e-3) / 1e12,
               "timing": "CUDA events around each kernel family of the step run kernel by "
                         "kernel (serialised), scaled by %.3f so the layer chain's families "
                         "add up to the timed graph step (side-stream families marked "
                         "overlapped)" % scale,
               "families": tab, "fused_phases_ms": parts or None})
    # end to end: the public call with pinned host tokens in, host logits out
    ht = torch.randint(0, S.vocab, (B,), dtype=torch.int32).pin_memory()
    hl = torch.empty(B, S.vocab).pin_memory()
    for _ in range(3):
        m.step(ht, logits=hl)
    reps = max(5, min(50, int(2000 / max(ms, 0.05))))
    t0 = time.perf_counter()
    for _ in range(reps):
        m.step(ht, logits=hl)
    e2e_s = dist.max(torch, (time.perf_counter() - t0) / reps)
    if B <= 8:  # fused step kernel + argmax
        launches = 2
    elif B >= 16:  # state split; per layer: Ws (side stream), prep, V, U, gate, Wz, LN planes,
        # Wc (tcgen05 GEMMs fed by planes their producers write); LN planes, head, 2 argmax
        launches = 8 * S.layers + 5
    else:  # per layer: prep, 5 SIMT GEMMs, gate, row stats; + stats, head, argmax
        launches = 8 * S.layers + 3
    res.update({
        "ms_per_step": ms,
        "value": seqs / (ms * 1e-3),
        "e2e": {"value": seqs / e2e_s, "unit": "tokens/s",
                "h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * S.vocab * 4,
                "call": "sn_abi_sunny_step (host tokens, host logits)"},
        "gpu_launches": launches * args.steps,
        "roofline": rl,
        "clocks": clk.summary(),
    })
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        ref_path = Path(td) / "ref.usnn"
        formats.write_usnn(ref_path, dequantised_weights(w) if quant else w)
        res["cpu_baseline"] = ref_sunny(ref_path, S, B)
    m.close()
    return res, None


def dequantised_weights(w):
    """USNQ semantics as fp32 weights: per-row INT8 codes times the row scale."""
    import copy
    from sunnynet_b200 import formats
    d = copy.deepcopy(w)

    def dq(a):
        q, sc = formats.quant_i8_rows(a)
        return (q.astype(np.float32) * sc[:, None]).astype(np.float32)

    for ly in d.layers:
        for k in ("V", "U", "Wz", "Wc", "Ws_eff"):
            ly[k] = dq(ly[k])
    d.head = dq(d.embed)  # the USNQ head is INT8; the embedding lookup stays fp32
    return d


def ref_sunny(path, S, B, budget_s=10.0):
    """Reference C runtime (oracle/_ref sn_step, B=1 per handle). B=1: one handle
    with the reference's recommended (physical-core) thread count. B>1: one
    single-threaded handle per physical core stepping concurrently (the C runtime
    has no batched step); throughput = tokens of all handles / wall time."""
    import ctypes
    import threading
    import oracle
    if oracle.ref_available():
        L, kind = oracle.ref_model(), "reference"
        load = lambda: L.sn_load(str(path).encode(), S.vocab, S.dim, S.inner, S.rank, S.taps,
                                 S.layers, S.group, 1)
        stepf = lambda h, t, buf: L.sn_step(h, int(t), buf)
        cores = max(1, int(L.sn_recommended_threads()))
    else:
        raise RuntimeError("oracle/_ref is not built; the CPU baseline needs the reference runtime")
    rng = np.random.default_rng(0)
    if B == 1:
        L.sn_set_threads(cores)
        h = load()
        buf = np.empty(S.vocab, np.float32)
        for t in rng.integers(0, S.vocab, 16):
            stepf(h, t, oracle.ptr(buf))
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            stepf(h, int(buf.argmax()), oracle.ptr(buf))
            n += 1
        dt = time.perf_counter() - t0
        L.sn_free(h)
        return {"value": n / dt, "unit": "tokens/s", "cores": cores, "kind": kind,
                "sample": f"{n} greedy B=1 sn_step calls after a 16-token prefill, "
                          f"{cores} OpenMP threads"}
    K = min(cores, B, 32)
    L.sn_set_threads(1)
    handles = [load() for _ in range(K)]
    counts = [0] * K
    stop = time.perf_counter() + budget_s

    def run(i):
        buf = np.empty(S.vocab, np.float32)
        p = oracle.ptr(buf)
        r = np.random.default_rng(i)
        for t in r.integers(0, S.vocab, 4):
            stepf(handles[i], t, p)
        while time.perf_counter() < stop:
            stepf(handles[i], int(buf.argmax()), p)
            counts[i] += 1

    t0 = time.perf_counter()
    ths = [threading.Thread(target=run, args=(i,)) for i in range(K)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    dt = time.perf_counter() - t0
    for h in handles:
        L.sn_free(h)
    return {"value": sum(counts) / dt, "unit": "tokens/s", "cores": K, "kind": kind,
            "sample": f"{sum(counts)} sn_step calls: {K} concurrent single-thread handles "
                      f"(the reference C runtime decodes B=1 per handle), ~{budget_s:.0f} s"}


def wl_c2(args, torch, dist, ours):
    return wl_sunny(args, torch, dist, ours, "c2", 256, False, 256, split=False)


def wl_c2b1(args, torch, dist, ours):
    return wl_sunny(args, torch, dist, ours, "c2", 1, False, 256, split=False)


def wl_c3(args, torch, dist, ours):
    res, base = wl_sunny(args, torch, dist, ours, "c3", 1024, True, 2048, split=True)
    if ours and dist.world == 1 and not args.no_sub_records and not args.ncu:
        # the metric's other batch sizes, on the same GPU in the same run
        subs = {}
        for name, fn in (("c2_b256", wl_c2), ("c2_b1", wl_c2b1)):
            r, _ = fn(args, torch, dist, True)
            subs[name] = {k: r[k] for k in ("config", "dtype", "value", "unit", "ms_per_step",
                                            "e2e", "roofline", "clocks", "gpu_launches",
                                            "cpu_baseline") if k in r}
        res["sub_records"] = subs
    return res, base


def wl_c5(args, torch, dist, ours):
    """Chunked prefill, BASELINE config 5 shape (L24 d1536 i2688 r960 V32000
    fp32). One step = one 256-token chunk for each of 8 sequences per GPU,
    continuing the same sequences (only the recurrent state is carried)."""
    from sunnynet_b200 import formats
    S = formats.SUNNY_PRESETS["c5"]
    B, Tc = 8, 256
    D, I, R, L = S.dim, S.inner, S.rank, S.layers
    mats = D * R + R * 2 * D + D * I + I * D + D * D
    flops = 2 * B * Tc * L * mats
    res = {"metric": "prefill tokens/s", "unit": "tokens/s", "higher_is_better": True,
           "dtype": "f32 (bf16x3 tensor-core split, fp32 accumulate)",
           "config": {"workload": f"c5 chunked prefill L{L} d{D} i{I} r{R} V{S.vocab} fp32",
                      "batch_per_gpu": B, "global_batch": B * dist.world, "chunk": Tc,
                      "step": "one 256-token chunk of every sequence",
                      "weights": "scaled-Gaussian random init (orthogonal QR at d2688 is "
                                 "minutes of CPU; same scale)",
                      "l2": "working set > L2"}}
    td = tempfile.mkdtemp(prefix="snbench5_")
    path = Path(td) / "m.usnn"
    formats.write_usnn(path, formats.random_sunny(S, seed=0, fast=True))
    if not ours:
        return res, ref_prefill(path, S)
    from sunnynet_b200 import _lib
    from sunnynet_b200._lib import check
    from sunnynet_b200.model import SunnyBatch
    lib = _lib.load()
    check(lib.sn_abi_cuda_set_stream(torch.cuda.current_stream().cuda_stream))
    m = SunnyBatch(path, B)
    check(lib.sn_abi_cuda_set_async(1))
    g = torch.Generator(device="cuda").manual_seed(dist.rank)
    toks = torch.randint(0, S.vocab, (B, Tc), generator=g, device="cuda", dtype=torch.int32)

    def step():
        m.prefill(toks, chunk=Tc, want_logits=False)

    with ClockSampler(dist.local) as clk:
        ms = timed_steps(torch, dist, step, args.steps, args.warmup)
        keep_busy(torch, step, inner=4)
    check(lib.sn_abi_cuda_profile(1))  # serialised family timing, scaled below
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    check(lib.sn_abi_cuda_profile(0))
    fams = _lib.profile_report()
    check(lib.sn_abi_cuda_set_async(0))
    peaks = measured_peaks()
    tab, scale, _ = family_table(fams, 2, ms)
    shapes = {"gemm_V": (R, D), "gemm_U": (2 * D, R), "gemm_Ws": (D, D), "gemm_Wz": (I, D),
              "gemm_Wc": (D, I)}
    dom = max((k for k in tab if k in shapes), key=lambda k: tab[k]["ms"])
    n_l, t_ms = tab[dom]["launches"], tab[dom]["ms"]
    n, k = shapes[dom]
    ff = 2 * B * Tc * n * k
    ach = ff / (t_ms / n_l * 1e-3) / 1e12
    rl = {"bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops_sustained"],
          "unit": "TFLOP/s", "frac": ach / peaks["bf16_tflops_sustained"],
          "peak_src": peaks["src"] + " (sustained bf16)", "kernel": dom, "launches": n_l,
          "avg_launch_us": t_ms / n_l * 1e3,
          "avg_launch_us_serialised": tab[dom]["serial_ms"] / n_l * 1e3,
          "alg_flops_per_launch": ff,
          "note": "achieved counts the fp32 product once; the bf16x3 split issues 3 MMAs",
          "traffic": profile_traffic(f"{dom}/c5"),
          "step_tflops": flops / (ms * 1e-3) / 1e12,
          "timing": "CUDA events around each kernel family of the step run kernel by "
                    "kernel (serialised), scaled by %.3f so the families add up to the "
                    "timed graph step" % scale,
          "families": tab}
    # end to end: host token ids in (pinned), host logits of the last position out
    ht = toks.cpu().pin_memory()
    hl = torch.empty(B, S.vocab).pin_memory()
    m.prefill(ht, chunk=Tc, logits=hl)
    reps = 5
    t0 = time.perf_counter()
    for _ in range(reps):
        m.prefill(ht, chunk=Tc, logits=hl)
    e2e_s = dist.max(torch, (time.perf_counter() - t0) / reps)
    # embedding gather; per layer LN rows, taps (writing V's input planes),
    # ring update, V (writing U's planes), U, gate (writing Wz's planes),
    # scan (writing Ws's input planes, the state entering each position), Ws,
    # Wz, LN of z into Wc's planes, Wc; the head's row statistics, input split
    # and contraction
    launches = 1 + L * 11 + 3
    res.update({"ms_per_step": ms, "value": B * Tc * dist.world / (ms * 1e-3),
                "e2e": {"value": B * Tc * dist.world / e2e_s, "unit": "tokens/s",
                        "h2d_bytes_per_step": B * Tc * 4, "d2h_bytes_per_step": B * S.vocab * 4,
                        "call": "sn_abi_sunny_prefill_chunked (host ids, host logits)"},
                "gpu_launches": launches * args.steps, "roofline": rl, "clocks": clk.summary()})
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = ref_prefill(path, S)
    m.close()
    return res, None


def ref_prefill(path, S, budget_s=15.0):
    """Reference C runtime prefill (sn_prefill = token-by-token sn_step,
    sunnynet.c:347-349) on one sequence, all physical cores."""
    import oracle
    if not oracle.ref_available():
        raise RuntimeError("oracle/_ref is not built; the CPU baseline needs the reference runtime")
    L = oracle.ref_model()
    cores = max(1, int(L.sn_recommended_threads()))
    L.sn_set_threads(cores)
    h = L.sn_load(str(path).encode(), S.vocab, S.dim, S.inner, S.rank, S.taps, S.layers, S.group, 1)
    buf = np.empty(S.vocab, np.float32)
    rng = np.random.default_rng(0)
    n, t0 = 0, time.perf_counter()
    toks = rng.integers(0, S.vocab, 4096).astype(np.int32)
    while time.perf_counter() - t0 < budget_s and n < len(toks):
        L.sn_step(h, int(toks[n]), oracle.ptr(buf))
        n += 1
    dt = time.perf_counter() - t0
    L.sn_free(h)
    return {"value": n / dt, "unit": "tokens/s", "cores": cores, "kind": "reference",
            "sample": f"{n} prompt tokens through sn_step (the reference prefill loop), "
                      f"{cores} OpenMP threads"}


def rwkv_step_cost(S, B, q4_bytes):
    """Algorithmic bytes / FLOPs of one RWKV-7 decode step: weights once,
    matrix state and token shift read+written, embedding rows, logits."""
    D, F, V, L = S.dim, S.ffn, S.vocab, S.layers
    Rw, Ra, Rv, Rg = S.ranks
    mats = 4 * D * D + D * (Rw + Ra + Rv + Rg) * 2 + 2 * D * F
    state = 2 * B * L * (S.n_head * S.head_size ** 2 + 2 * D) * 4
    return q4_bytes + state + B * D * 4 + B * V * 4, 2 * B * (L * mats + V * D)


def rwkv_launches(S, B, block=128):
    """Kernels one greedy RWKV-7 step launches (rwkv7.cu enqueue_rk + argmax):
    a W4A8 matrix is one weight-streaming launch below 16 sequences, or a
    quantise + tensor-core launch when its shape suits the tensor cores; the
    first-stage projections of a layer share one such pair when all suit."""
    D, F = S.dim, S.ffn
    Rw, Ra, Rv, Rg = S.ranks
    if B == 1:  # one sequence: the fused persistent step kernel, then the two argmax kernels
        return 3

    def tc(K, N):
        return B >= 16 and N >= 32 and K % 128 == 0 and block in (32, 64, 128)

    def mm(K, N):
        return 2 if tc(K, N) else 1

    n = 1  # embed + LN0
    for l in range(S.layers):
        first = [(D, D)] * 3 + [(D, Rw), (D, Ra), (D, Rg)] + ([(D, Rv)] if l > 0 else [])
        grouped = all(tc(K, N) for K, N in first)
        small = B <= 8 and all(K % block == 0 for K, N in first)  # one SIMT group launch
        n += 1 + (2 if grouped else 1 if small else sum(mm(K, N) for K, N in first))  # prep + stage 1
        # LoRA second stages: ranks below a quantisation block stay fp32 and are
        # folded into the mix kernel; g2 (and any quantised one) is a contraction
        fp32 = [r % block != 0 for r in (Rw, Ra, Rv)]
        if all(fp32):
            n += mm(Rg, D) + 1  # g2, fused LoRA + mix
        else:
            n += mm(Rw, D) + mm(Ra, D) + mm(Rg, D) + (mm(Rv, D) if l > 0 else 0) + 1
        n += 1 + mm(D, D) + 1 + mm(D, F) + mm(F, D)  # heads, out, cmix prep, ffn
    return n + 2 + 2  # final LN + head (fp32), argmax partials + final


def wl_rwkv(args, torch, dist, ours, B):
    from sunnynet_b200 import formats
    S = formats.RWKV_PRESETS["c4"]
    td = tempfile.mkdtemp(prefix="snbench4_")
    path = Path(td) / "c4.q4g.bin"
    w = formats.random_rwkv(S, 0)
    info = formats.write_krwk(path, w, quant="q4g", group=128)
    step_bytes, step_flops = rwkv_step_cost(S, B, info["bytes"] - S.vocab * S.dim * 4)
    res = {"metric": "decode tokens/s", "unit": "tokens/s", "higher_is_better": True,
           "dtype": "int4w-a8 (W4A8) + f32",
           "config": {"workload": f"c4 RWKV-7 L{S.layers} D{S.dim} H{S.n_head}x{S.head_size} "
                                  f"F{S.ffn} V{S.vocab}, INT4 group 128 fp16 scales",
                      "batch_per_gpu": B, "global_batch": B * dist.world,
                      "decode": "greedy", "l2": "flushed between steps"
                      if step_bytes < 2 * (126 << 20) else "working set > L2"}}
    ref_blob = Path(td) / "c4.q4v3.bin"  # the reference's only INT4 format (block 64, fp32 scales)
    if not ours:
        formats.write_krwk(ref_blob, w, quant="q4")
        return res, ref_rwkv(ref_blob, S, B)
    from sunnynet_b200 import _lib
    from sunnynet_b200._lib import check
    from sunnynet_b200.rwkv7 import Rwkv7Batch
    lib = _lib.load()
    check(lib.sn_abi_cuda_set_stream(torch.cuda.current_stream().cuda_stream))
    m = Rwkv7Batch(path, B)
    check(lib.sn_abi_cuda_set_async(1))
    g = torch.Generator(device="cuda").manual_seed(dist.rank)
    cur = torch.randint(0, S.vocab, (B,), generator=g, device="cuda", dtype=torch.int32)
    for _ in range(8):
        m.step_argmax(cur, out=cur)

    def step():
        m.step_argmax(cur, out=cur)

    flushbuf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    flush = flushbuf.zero_ if step_bytes < 2 * (126 << 20) else None
    with ClockSampler(dist.local) as clk:
        ms = timed_steps(torch, dist, step, args.steps, args.warmup, flush=flush)
        keep_busy(torch, step)
    check(lib.sn_abi_cuda_profile(1))  # serialised family timing, scaled below
    for _ in range(3):
        if flush:
            flush()
        step()
    torch.cuda.synchronize()
    check(lib.sn_abi_cuda_profile(0))
    fams = _lib.profile_report()
    check(lib.sn_abi_cuda_set_async(0))
    tab, scale, _ = family_table(fams, 3, ms)
    dom = max(tab, key=lambda k: tab[k]["ms"])
    n_l, t_ms = tab[dom]["launches"], tab[dom]["ms"]
    peaks = measured_peaks()
    step_gbs = step_bytes / (ms * 1e-3) / 1e9
    if dom == "rk_heads":  # per launch: one layer's matrix states read + written
        fb = 2 * B * S.n_head * S.head_size ** 2 * 4
        ach = fb / (t_ms / n_l * 1e-3) / 1e9
    else:
        fb, ach = None, None
    rl = {"bound": "hbm", "achieved": ach if ach else step_gbs, "peak": peaks["hbm_gbs"],
          "unit": "GB/s", "peak_src": peaks["src"], "kernel": dom, "launches": n_l,
          "avg_launch_us": t_ms / n_l * 1e3,
          "avg_launch_us_serialised": tab[dom]["serial_ms"] / n_l * 1e3,
          "alg_bytes_per_launch": fb,
          "achieved_is": "dominant kernel" if ach else (
              "whole step (one fused kernel)" if dom == "rk_fused"
              else "whole step (dominant is a GEMV family)"),
          "traffic": profile_traffic(f"{dom}/c4/B{B}"), "step_alg_bytes": step_bytes,
          "step_alg_flops": step_flops, "step_hbm_gbs": step_gbs,
          "timing": "CUDA events around each kernel family of the step run kernel by "
                    "kernel (serialised), scaled by %.3f so the families add up to the "
                    "timed graph step" % scale,
          "families": tab}
    rl["frac"] = rl["achieved"] / rl["peak"]
    ht = torch.randint(0, S.vocab, (B,), dtype=torch.int32).pin_memory()
    hl = torch.empty(B, S.vocab).pin_memory()
    for _ in range(2):
        m.step(ht, logits=hl)
    reps = max(5, min(40, int(2000 / max(ms, 0.05))))
    t0 = time.perf_counter()
    for _ in range(reps):
        m.step(ht, logits=hl)
    e2e_s = dist.max(torch, (time.perf_counter() - t0) / reps)
    res.update({"ms_per_step": ms, "value": B * dist.world / (ms * 1e-3),
                "e2e": {"value": B * dist.world / e2e_s, "unit": "tokens/s",
                        "h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * S.vocab * 4,
                        "call": "sn_abi_rwkv7_step_batch (host ids, host logits)"},
                "gpu_launches": rwkv_launches(S, B) * args.steps, "roofline": rl,
                "clocks": clk.summary()})
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        formats.write_krwk(ref_blob, w, quant="q4")
        res["cpu_baseline"] = ref_rwkv(ref_blob, S, B)
    m.close()
    return res, None


def ref_rwkv(path, S, B, budget_s=10.0):
    """Reference C runtime sn_rk_step on its INT4 blob (block 64, fp32 scales:
    the only INT4 format rwkv7.c reads). B=1: one handle; B>1: one handle per
    physical core stepping concurrently (the C runtime is B=1 per handle)."""
    import threading
    import oracle
    if not oracle.ref_available():
        raise RuntimeError("oracle/_ref is not built; the CPU baseline needs the reference runtime")
    L = oracle.ref_abi()
    cores = max(1, int(oracle.ref_model().sn_recommended_threads()))
    K = 1 if B == 1 else min(cores, B, 32)
    L.sn_set_threads(cores if B == 1 else 1)
    hs = [L.sn_rk_load(str(path).encode()) for _ in range(K)]
    counts = [0] * K
    stop = time.perf_counter() + budget_s

    def run(i):
        buf = np.empty(S.vocab, np.float32)
        p = oracle.ptr(buf)
        L.sn_rk_step(hs[i], 1 + i, p)
        while time.perf_counter() < stop:
            L.sn_rk_step(hs[i], int(buf.argmax()), p)
            counts[i] += 1

    t0 = time.perf_counter()
    ths = [threading.Thread(target=run, args=(i,)) for i in range(K)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    dt = time.perf_counter() - t0
    for h in hs:
        L.sn_rk_free(h)
    return {"value": sum(counts) / dt, "unit": "tokens/s", "cores": cores if K == 1 else K,
            "kind": "reference",
            "sample": f"{sum(counts)} sn_rk_step calls on the reference INT4 blob (block 64), "
                      f"{K} handle(s), ~{budget_s:.0f} s"}


WORKLOADS = {"c1": wl_c1, "c2": wl_c2, "c2b1": wl_c2b1, "c3": wl_c3, "c5": wl_c5,
             "c4": lambda a, t, d, ours: wl_rwkv(a, t, d, ours, 64),
             "c4b1": lambda a, t, d, ours: wl_rwkv(a, t, d, ours, 1),
             "c4b512": lambda a, t, d, ours: wl_rwkv(a, t, d, ours, 512)}
SCALING = {"c3": "strong"}
DEFAULT_CONFIG = "c3"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub-records", action="store_true",
                    help="default config only: skip the c2 B=256 / B=1 sub-records")
    ap.add_argument("--prefill-tokens", type=int, default=None,
                    help="SunnyNet decode configs: prompt length before the timed steps")
    ap.add_argument("--ncu", action="store_true",
                    help="for a profiler's launch list: the prefill, W warm-up and K timed "
                         "steps only (no clock loop, family timing, e2e or CPU baseline)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    import torch
    dist = Dist()
    if args.impl == "reference":
        if dist.rank != 0:
            return 0
        res, base = WORKLOADS[args.config](args, torch, dist, ours=False)
        res.update({"impl": "reference", "value": base["value"], "n_gpus": args.gpus,
                    "steps": args.steps, "warmup": args.warmup,
                    "scaling": SCALING.get(args.config, "weak"),
                    "vs_baseline": None, "data": "synthetic", "cpu_baseline": base,
                    "e2e": {"value": base["value"], "unit": base["unit"],
                            "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        print(json.dumps(res))
        return 0
    dist.init(torch)
    try:
        res, _ = WORKLOADS[args.config](args, torch, dist, ours=True)
        res.update({"n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
                    "scaling": SCALING.get(args.config, "weak"), "vs_baseline": None,
                    "data": "synthetic (seeded random-init weights and token ids)"})
        if dist.rank == 0:
            print(json.dumps(res))
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
