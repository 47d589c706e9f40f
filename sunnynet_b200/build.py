"""Build libsunnynet_cuda.so in-tree with nvcc for sm_100a.

    python -m sunnynet_b200.build [--force] [--verbose]

The library links the CUDA runtime statically and exports only the C ABI
declared in include/*.h (no torch types cross it).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
BUILD = PKG / "_build"
LIB = PKG / "libsunnynet_cuda.so"

SOURCES = ["runtime.cu", "abi.cu", "recur.cu", "quant4.cu", "gemm.cu", "tc_gemm.cu", "sunny.cu",
           "rwkv7.cu", "scan_noalloc.cu", "sunny_fused.cu", "w4a8_tc.cu", "argmax.cu",
           "train.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _headers():
    return list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in _headers())


def _compile(src: Path, obj: Path, extra, verbose: bool):
    cmd = [nvcc()] + ARCH + FLAGS + list(extra) + ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr[-4000:]}")
    if verbose and r.stderr:
        print(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, extra=()) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(o, s)]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            list(ex.map(lambda so: _compile(so[0], so[1], extra, verbose), todo))
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        # no -lcuda: driver entry points are resolved at run time, so the
        # library also loads (and answers the ABI queries) on GPU-less hosts
        cmd = [nvcc()] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs] + [
            "-Xlinker", "--no-undefined"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print register/smem usage")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas else []
    p = build(force=a.force or a.ptxas, verbose=a.verbose or a.ptxas, extra=extra)
    print(p)


if __name__ == "__main__":
    sys.exit(main())
