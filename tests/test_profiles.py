"""The committed ncu summaries the bench reads its `roofline.traffic` from:
each gives the command that made it (ncu with the clocks left alone, on
committed files only), and each traffic figure parses as the bytes of one
launch that `bench.py` looks up for its dominant kernels."""
from __future__ import annotations

import importlib.util
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PROFILES = sorted((ROOT / "profiles").glob("*.md"))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_every_summary_names_its_command():
    assert PROFILES
    for f in PROFILES:
        t = f.read_text()
        assert "ncu " in t, f.name
        assert "--clock-control none" in t, f.name
        assert "_work/" not in t, f.name


def test_traffic_figures_parse_and_resolve():
    keys = {}
    for f in PROFILES:
        for m in re.finditer(r"traffic_bytes_per_launch\[(.+?)\]:\s*([0-9.eE+]+)", f.read_text()):
            assert m.group(1) not in keys, m.group(1)  # one figure per kernel and workload
            keys[m.group(1)] = float(m.group(2))
    assert all(v > 0 for v in keys.values())
    b = _bench()
    for k in ("rk_fused/c4/B1", "gemm_Wc/c3/B1024", "fused_step/c2/B1"):
        assert b.profile_traffic(k) == keys[k], k
    assert b.profile_traffic("no_such_kernel/c0") is None
