"""Tensor-parallel sharding (the multi-GPU configs 2-4): shards cut
from the packed streams decode to exactly the matching slice of the
original matrix, and the sharded layer's collectives (gloo ranks on CPU
here; NCCL on GPUs) reassemble the unsharded product.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import cases
import se12_oracle as oracle


def to_tensor(s: oracle.Streams):
    from se12_b200.format import make_tensor

    return make_tensor(s.rows, s.cols, s.codebook, s.sm, s.ec, s.esc, s.fallback_bitmap, s.fallback_raw)


def to_streams(t) -> oracle.Streams:
    return oracle.Streams(rows=t.rows, cols=t.cols, codebook=t.codebook, sm=t.sm, ec=t.ec, esc=t.esc,
                          fallback_bitmap=t.fallback_bitmap, fallback_raw=t.fallback_raw)


SHAPES = [
    ("random_bits", 160, 2560),   # many fallback tiles
    ("synthetic", 272, 2304),     # escapes, K % 1024 != 0
    ("synthetic", 48, 300),       # padded rows and columns
    ("concentrated", 64, 1024),
]


def matrix(kind, rows, cols):
    if kind == "random_bits":
        bits = np.random.default_rng(11).integers(0, 1 << 16, size=rows * cols, dtype=np.uint32).astype(np.uint16)
    elif kind == "synthetic":
        bits, _, _ = cases.synthetic_weights(rows, cols, seed=rows, outlier_rate=5e-3, outlier_scale=512.0)
    else:
        bits, _, _ = cases.concentrated(rows, cols, 3)
    bits = np.asarray(bits, dtype=np.uint16)
    return bits.reshape(rows, cols), oracle.encode(bits, rows, cols)


@pytest.mark.parametrize("kind,rows,cols", SHAPES)
@pytest.mark.parametrize("parts", [1, 2, 3])
def test_row_and_column_shards_decode_to_slices(kind, rows, cols, parts):
    from se12_b200.sharding import col_range, row_range, shard_cols, shard_rows

    full, streams = matrix(kind, rows, cols)
    t = to_tensor(streams)
    tr, tc = -(-rows // 16), -(-cols // 256)
    if parts <= tr:
        got_rows = []
        for r in range(parts):
            a, b = row_range(rows, parts, r)
            shard = to_streams(shard_rows(t, parts, r))
            assert (shard.rows, shard.cols) == (b - a, cols)
            assert shard.codebook == streams.codebook
            assert np.array_equal(oracle.decode(shard), full[a:b])
            got_rows.append(b - a)
        assert sum(got_rows) == rows
    if parts <= tc:
        for r in range(parts):
            a, b = col_range(cols, parts, r)
            shard = to_streams(shard_cols(t, parts, r))
            assert (shard.rows, shard.cols) == (rows, b - a)
            assert np.array_equal(oracle.decode(shard), full[:, a:b])


def test_too_many_shards_is_refused():
    from se12_b200.sharding import shard_rows

    _, streams = matrix("synthetic", 48, 300)
    with pytest.raises(ValueError):
        shard_rows(to_tensor(streams), 4, 0)  # 3 tile rows


def test_megatron_plan():
    from se12_b200.sharding import megatron_plan

    assert megatron_plan("model.layers.3.self_attn.q_proj") == "rows"
    assert megatron_plan("model.layers.3.self_attn.o_proj") == "cols"
    assert megatron_plan("model.layers.3.mlp.down_proj") == "cols"
    assert megatron_plan("model.layers.3.mlp.up_proj") == "rows"
    assert megatron_plan("lm_head") == "rows"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    import torch.distributed as dist

    from se12_b200.sharding import ShardedLinear, shard_cols, shard_rows

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        full, streams = matrix("synthetic", 272, 2304)
        t = to_tensor(streams)
        w = torch.from_numpy(oracle.bits_to_float32(full.reshape(-1)).reshape(272, 2304)).double()
        x = torch.from_numpy(np.random.default_rng(5).normal(size=(3, 2304))).double()
        want = x @ w.T
        errs = []
        for kind, cut in (("rows", shard_rows), ("cols", shard_cols)):
            part = to_streams(cut(t, world, rank))
            wl = torch.from_numpy(oracle.bits_to_float32(oracle.decode(part).reshape(-1)).reshape(part.rows, part.cols)).double()
            layer = ShardedLinear(kind, 272, 2304, world, rank, local=lambda xl, wl=wl: xl.double() @ wl.T)
            got = layer(x.float()).double()
            errs.append(float((got - want).abs().max() / want.abs().max()))
        torch.save(errs, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_sharded_layer_collectives_on_gloo(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path / "errs")), nprocs=world, join=True)
    for r in range(world):
        errs = torch.load(tmp_path / f"errs.{r}")
        assert max(errs) < 1e-5, errs
