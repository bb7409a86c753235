"""bench.py's output contract, checked without a GPU: the reference arm (the
reference's CPU path, restated in the oracle, on the host cores) prints one
JSON line with the keys a driver reads, and ranks other than 0 print
nothing; the per-step percentile helper of the GPU arm; the tensor-parallel
legs' shards (inputs of each matrix's width, collectives per split)."""

from __future__ import annotations

import json
import os
import pathlib
import subprocess
import sys

import pytest

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


@pytest.mark.parametrize("split", ["megatron", "rows"])
@pytest.mark.parametrize("world", [1, 2, 8])
def test_tensor_parallel_ops_read_inputs_of_their_width(monkeypatch, split, world):
    """tp_build's shards (weights faked on the CPU): every op's x has its
    matrix's columns, and the collectives follow the split: Megatron
    all-reduces o/down and all-gathers the LM head; the row split
    all-gathers every output."""
    import torch

    import bench
    import se12_b200.codec as codec
    import se12_b200.device as device
    from se12_b200.shapes import CONFIGS

    class Fake:
        def __init__(self, rows, cols):
            self.rows, self.cols, self.byte_size = rows, cols, rows * cols

    monkeypatch.setattr(codec, "encode_device", lambda w: Fake(*w.shape))
    monkeypatch.setattr(device.DeviceSe12Matrix, "concatenate",
                        staticmethod(lambda parts: Fake(sum(p.rows for p in parts), parts[0].cols)))
    monkeypatch.setattr(bench, "synthetic_bf16", lambda torch_, r, c, seed, dev, **kw: torch.empty(r, c))
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    shapes = CONFIGS["gemma2-9b"]
    ops, _ = bench.tp_build(torch, shapes, 2, 3, world, world - 1, torch.device("cpu"), split=split)
    assert len(ops) == 2 * 4 + 1
    for op in ops:
        assert tuple(op.x.shape) == (3, op.m.cols)
        if split == "rows":
            assert op.plan == "rows" and op.coll == "all_gather"
        elif op.names[0] in ("o_proj", "down_proj"):
            assert op.plan == "cols" and op.coll == "all_reduce"
        else:
            assert op.plan == "rows" and op.coll == ("all_gather" if op.names[0] == "lm_head" else None)
