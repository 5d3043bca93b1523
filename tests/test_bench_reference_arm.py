"""bench.py --impl reference without a GPU: the reference arm times the CPU reference of this
path (the literal C restatement of DeformConvCPU.run, DeformConv.swift:75-166) on the host
cores and prints one JSON line with the fields the benchmark contract asks of that arm."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "Mpx/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["gpu_launches"] == 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"] == {"value": d["value"], "unit": "Mpx/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "config 4" in d["metric"]


def test_clock_sampler_keeps_the_timed_region():
    """The bench's clock record comes from nvidia-smi samples taken inside the timed region (by
    nvidia-smi's own timestamps), median SM clock and every slowdown reason seen there; with no
    sample inside a very short region it falls back to all samples and says so."""
    import datetime
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", REPO / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    t0 = datetime.datetime(2026, 1, 2, 3, 4, 5)

    def line(ms, sm, reasons=("Not Active",) * 4):
        ts = (t0 + datetime.timedelta(milliseconds=ms)).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
        return ", ".join([ts, "0", str(sm), "1965", "700.0", "0x0", *reasons])

    lines = [line(0, 1100), line(50, 1965), line(100, 1965, ("Not Active",) * 3 + ("Active",)), line(150, 1950),
             line(400, 1200), "garbage"]
    base = t0.timestamp()
    got = bench.ClockSampler.summarize(lines, window=(base + 0.04, base + 0.16))
    assert got["samples_in_timed_region"] == 3 and got["samples"] == 3
    assert got["sm_mhz"] == 1965.0 and got["sm_max_mhz"] == 1965.0
    assert got["reasons"] == ["sw_power_cap"]
    fallback = bench.ClockSampler.summarize(lines, window=(base + 0.2, base + 0.21))
    assert fallback["samples_in_timed_region"] == 0 and fallback["samples"] == 5
    assert bench.ClockSampler.summarize([], window=None)["sm_mhz"] is None
