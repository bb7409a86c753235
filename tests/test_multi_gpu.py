"""Tensor-parallel SE12 layers on real GPUs over NCCL (two ranks, one GPU
each): row shards + all-gather and column shards + all-reduce reproduce the
fp64 oracle within the GEMV tolerance. Skipped with fewer than two GPUs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import cases
import se12_oracle as oracle

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    import datetime

    import torch.distributed as dist

    from se12_b200.format import make_tensor
    from se12_b200.sharding import shard_matrix

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        rows, cols = 1040, 4608  # 65 tile rows: uneven row shards
        bits, _, _ = cases.synthetic_weights(rows, cols, seed=8, outlier_rate=2e-3, outlier_scale=256.0)
        s = oracle.encode(np.asarray(bits, dtype=np.uint16), rows, cols)
        t = make_tensor(s.rows, s.cols, s.codebook, s.sm, s.ec, s.esc, s.fallback_bitmap, s.fallback_raw)
        xb = oracle.bf16_round(np.random.default_rng(4).normal(size=(3, cols)).astype(np.float32))
        y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
        errs = []
        for kind in ("rows", "cols"):
            layer = shard_matrix(t, kind, world, rank, device=f"cuda:{rank}")
            y = layer(x).cpu().numpy()
            errs.append(oracle.max_relative_error(y, y64))
        torch.cuda.synchronize()
        torch.save(errs, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_row_and_column_sharded_layers_over_nccl(tmp_path):
    import torch.multiprocessing as mp

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_rank_main, args=(2, _free_port(), str(tmp_path / "errs")), nprocs=2, join=True)
    for r in range(2):
        errs = torch.load(tmp_path / f"errs.{r}")
        assert max(errs) <= TOLERANCE, errs
