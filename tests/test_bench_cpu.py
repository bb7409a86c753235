"""bench.py's output contract, checked without a GPU: the reference arm (the
reference's CPU path, restated in the oracle, on the host cores) prints one
JSON line with the keys a driver reads, and ranks other than 0 print
nothing; the per-step percentile helper of the GPU arm."""

from __future__ import annotations

import json
import os
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent


def run_bench(*args, env=None):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True, timeout=600,
                          cwd=ROOT, env={**os.environ, **(env or {})})


def test_reference_arm_prints_the_contract_line():
    res = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [line for line in res.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    import bench

    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "GB/s"
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1 and d["higher_is_better"] is True
    assert d["scaling"] == "weak" and d["vs_baseline"] is None and d["data"] == "synthetic"
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"]
    assert "workload" in d["config"]


def test_reference_arm_other_ranks_print_nothing():
    res = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1", env={"RANK": "1", "WORLD_SIZE": "2"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert not [line for line in res.stdout.splitlines() if line.startswith("{")]


def test_step_percentiles():
    import bench

    p = bench.step_percentiles([float(v) for v in range(10, 0, -1)])
    assert (p["p10"], p["median"], p["p90"], p["steps"]) == (2.0, 6.0, 9.0, 10)
    assert bench.step_percentiles([3.5]) == {"p10": 3.5, "median": 3.5, "p90": 3.5, "steps": 1, "rank": "0"}
    assert bench.step_percentiles([]) is None
