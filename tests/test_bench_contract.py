"""The JSON line of `bench.py --impl reference` (the reference's own CPU operators on the host cores): one line with the
keys the driver reads, the same metric, unit and config as the GPU arm (the same suite: ops, shapes, element types and
bytes a step), and the reference-arm extras (impl, cpu_baseline, e2e with no host<->device bytes). Also the clock
sampler's summary on a machine without a GPU. Runs on the CPU in about ten seconds."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("HBM GB/s") and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] >= 3 and d["scaling"] in ("weak", "strong")
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"] == "vox-hotpath-suite"
    sys.path.insert(0, str(ROOT))
    import bench

    assert d["config"] == bench.suite_config(1 << 27)  # the GPU arm's default config, like for like
    assert len(d["config"]["ops"]) == 20 and d["config"]["bytes_per_step_per_gpu"] == sum(b for _, b, _ in bench.suite_model(1 << 27))
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["cores"] >= 1 and cb["kind"] in ("reference", "port")
    assert isinstance(cb["sample"], str) and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_clock_sampler_summary_without_samples():
    """With no GPU (or no samples) the summary still has the driver's keys, with no clock and no reason."""
    sys.path.insert(0, str(ROOT))
    import bench

    c = bench.ClockSampler(0)
    s = c.summary()
    assert set(s) >= {"sm_mhz", "sm_max_mhz", "reasons", "samples"} and s["samples"] == 0 and s["reasons"] == []
