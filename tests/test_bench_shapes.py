"""Parity on the shapes the benchmark times (Gemma-2-2B decode step, batch 1,
2, 4, 8 and 16), through the same launch choice the benchmark makes: the
grouped q/k/v (3 segments) and gate/up (2 segments) matrices, o, k/v alone,
down and the 256000-row LM head (AC-011 of the reference's fused-GEMV spec,
.spec/features/fused-decode-gemv/spec.md:82-87: every distinct linear
weight shape, the tied embedding used as LM head included).

The weights are the benchmark's own synthetic distribution (bench.py:
N(0, 0.02) BF16, 0.01 % x64 outliers, 0.1 % +-0), drawn and packed on the
GPU. SE12 is lossless, so the fp64 reference is the original BF16 matrix
times x in float64 on the host (the oracle's gemv_fp64); for the LM head it
covers 4096 rows spread over the whole matrix (every CTA's share),
elsewhere every row. Metric and bound: max |y - y64| / max(|y64|, 1) <= 1e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import se12_oracle as oracle

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-3
BATCHES = (1, 2, 4, 8, 16)

# name -> member shapes (rows, cols); several members form one segmented matrix
SHAPES = {
    "qkv_grouped": [(2048, 2304), (1024, 2304), (1024, 2304)],
    "k_proj": [(1024, 2304)],
    "o_proj": [(2304, 2048)],
    "gate_up_grouped": [(9216, 2304), (9216, 2304)],
    "down_proj": [(2304, 9216)],
    "lm_head": [(256000, 2304)],
}
SAMPLE_ROWS = 4096


@pytest.fixture(scope="module", autouse=True)
def library():
    from se12_b200 import _build

    _build.build()
    torch.cuda.set_device(0)
    yield
    _cache.clear()
    torch.cuda.empty_cache()


_cache: dict = {}


def bench_matrix(name):
    """(device matrix, host float64 weights of the sampled rows, sampled row ids)."""
    if name in _cache:
        return _cache[name]
    import bench
    from se12_b200.codec import encode_device
    from se12_b200.device import DeviceSe12Matrix

    dev = torch.device("cuda", 0)
    parts, dense = [], []
    for j, (rows, cols) in enumerate(SHAPES[name]):
        w = bench.synthetic_bf16(torch, rows, cols, 7000 + 17 * j + rows, dev)
        parts.append(encode_device(w))
        dense.append(w)
    m = DeviceSe12Matrix.concatenate(parts) if len(parts) > 1 else parts[0]
    w = torch.cat(dense) if len(dense) > 1 else dense[0]
    if m.rows > SAMPLE_ROWS:
        g = torch.Generator().manual_seed(5)
        spread = torch.linspace(0, m.rows - 1, SAMPLE_ROWS // 2).long()
        extra = torch.randint(0, m.rows, (SAMPLE_ROWS // 2,), generator=g)
        ids = torch.unique(torch.cat([spread, extra, torch.tensor([0, m.rows - 1])]))
    else:
        ids = torch.arange(m.rows)
    w64 = w[ids.to(dev)].float().cpu().double().numpy()
    del dense, w
    _cache[name] = (m, w64, ids.numpy())
    return _cache[name]


def activations(batch, cols, seed):
    x = np.random.default_rng(seed).normal(0.0, 1.0, size=(batch, cols)).astype(np.float32)
    return oracle.bf16_round(x)


@pytest.mark.parametrize("batch", BATCHES)
@pytest.mark.parametrize("name", list(SHAPES))
def test_bench_shape_matches_fp64(name, batch):
    m, w64, ids = bench_matrix(name)
    xb = activations(batch, m.cols, seed=batch * 31 + m.rows)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = m.gemv(x).cpu().numpy()[:, ids]
    y64 = oracle.bits_to_float32(xb).astype(np.float64) @ w64.T
    err = oracle.max_relative_error(y, y64)
    assert err <= TOLERANCE, f"{name} batch {batch}: max rel err {err:.3e}"


def test_bench_shapes_reach_the_benchmark_layouts():
    """The matrices above run the launch configurations the benchmark uses
    for them (so the parity covers the timed kernels): on a 148-SM B200 the
    LM head takes the wide layout at batch 1, and the down projection (144
    tile rows, one wave) 8-tile stages in one CTA per SM."""
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("launch choices are stated for 148 SMs")
    assert bench_matrix("lm_head")[0].launch_config(1)["wide"] == 1
    down = bench_matrix("down_proj")[0].launch_config(1)
    assert down["wide"] == 0 and down["stage_tiles"] == 8 and down["ctas_per_sm"] == 1
    assert bench_matrix("gate_up_grouped")[0].launch_config(1)["stage_tiles"] == 8
