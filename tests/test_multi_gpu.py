"""Tensor-parallel SE12 layers on real GPUs (2, 4 and 8 ranks, one GPU
each): row shards + NCCL all-gather, column shards + NCCL all-reduce, and
column shards whose all-reduce is fused into the GEMV reproduce the fp64
oracle within the GEMV tolerance. A world size is skipped when fewer GPUs
are visible.
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


WORLDS = (2, 4, 8)


def _need(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


@pytest.mark.parametrize("world", WORLDS)
def test_row_and_column_sharded_layers_over_nccl(tmp_path, world):
    import torch.multiprocessing as mp

    _need(world)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path / "errs")), nprocs=world, join=True)
    for r in range(world):
        errs = torch.load(tmp_path / f"errs.{r}")
        assert max(errs) <= TOLERANCE, errs


def _allreduce_main(rank, world, port, result_path):
    import datetime

    import torch.distributed as dist

    from se12_b200.device import device_status
    from se12_b200.format import make_tensor
    from se12_b200.peers import PeerGroup
    from se12_b200.sharding import col_range, shard_matrix

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    out = {}
    try:
        mats = {}
        for name, rows, cols, seed in (("a", 1040, 4608, 8), ("b", 2304, 2048, 9)):  # 65 tile rows: a ragged last row
            bits, _, _ = cases.synthetic_weights(rows, cols, seed=seed, outlier_rate=2e-3, outlier_scale=256.0)
            s = oracle.encode(np.asarray(bits, dtype=np.uint16), rows, cols)
            t = make_tensor(s.rows, s.cols, s.codebook, s.sm, s.ec, s.esc, s.fallback_bitmap, s.fallback_raw)
            mats[name] = (bits, rows, cols, t)
        peers = PeerGroup(rows_cap=2304)
        layers = {n: shard_matrix(t, "cols", world, rank, device=f"cuda:{rank}", peers=peers) for n, (_, _, _, t) in mats.items()}
        errs, same = [], []
        # calls in a row, alternating matrices and batch sizes (20: two calls of 16 + 4)
        for call, (name, batch) in enumerate((("a", 1), ("b", 3), ("a", 16), ("b", 20), ("a", 2))):
            bits, rows, cols, _ = mats[name]
            xb = oracle.bf16_round(np.random.default_rng(call).normal(size=(batch, cols)).astype(np.float32))
            x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
            y = layers[name](x)
            y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
            errs.append(oracle.max_relative_error(y.cpu().numpy(), y64))
            everyone = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(everyone, y)
            same.append(all(torch.equal(everyone[0], e) for e in everyone))
        # the same calls from a CUDA graph: the call counter lives in device memory
        bits, rows, cols, _ = mats["b"]
        xb = oracle.bf16_round(np.random.default_rng(99).normal(size=(4, cols)).astype(np.float32))
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
        c0, c1 = col_range(cols, world, rank)
        xs = x[:, c0:c1].contiguous()
        y = torch.empty(4, rows, device="cuda")
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            peers.gemv_allreduce(layers["b"].matrix, xs, y)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            peers.gemv_allreduce(layers["b"].matrix, xs, y)
            peers.gemv_allreduce(layers["b"].matrix, xs, y)
        y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
        for _ in range(3):
            y.zero_()
            graph.replay()
            torch.cuda.synchronize()
            errs.append(oracle.max_relative_error(y.cpu().numpy(), y64))
        del graph
        torch.cuda.synchronize()
        out = {"errs": errs, "same": same, "status": device_status()}
        peers.close()
    finally:
        torch.save(out, f"{result_path}.{rank}")
        dist.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_fused_gemv_allreduce_over_peer_memory(tmp_path, world):
    """Column shards whose GEMV and all-reduce are one kernel (peer memory,
    no NCCL on the data path): within 1e-3 of the fp64 oracle, the same bits
    on every rank, over calls in a row and from a replayed CUDA graph."""
    import torch.multiprocessing as mp

    _need(world)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_allreduce_main, args=(world, _free_port(), str(tmp_path / "ar")), nprocs=world, join=True)
    for r in range(world):
        res = torch.load(tmp_path / f"ar.{r}")
        assert res["status"] == 0, res
        assert max(res["errs"]) <= TOLERANCE, res["errs"]
        assert all(res["same"]), res["same"]


def _lost_peer_main(rank, world, port, result_path):
    import datetime
    import time

    import torch.distributed as dist

    from se12_b200.device import STATUS_WAIT_TIMEOUT, device_status, set_wait_limit_ns
    from se12_b200.format import make_tensor
    from se12_b200.peers import PeerGroup
    from se12_b200.sharding import shard_matrix

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    out = {}
    try:
        rows, cols = 1040, 4608
        bits, _, _ = cases.synthetic_weights(rows, cols, seed=8)
        s = oracle.encode(np.asarray(bits, dtype=np.uint16), rows, cols)
        t = make_tensor(s.rows, s.cols, s.codebook, s.sm, s.ec, s.esc, s.fallback_bitmap, s.fallback_raw)
        peers = PeerGroup(rows_cap=rows)
        layer = shard_matrix(t, "cols", world, rank, device=f"cuda:{rank}", peers=peers)
        xb = oracle.bf16_round(np.random.default_rng(1).normal(size=(1, cols)).astype(np.float32))
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
        y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
        good = oracle.max_relative_error(layer(x).cpu().numpy(), y64)  # every rank calls: fine
        torch.cuda.synchronize()
        dist.barrier()
        set_wait_limit_ns(100_000_000)
        elapsed = None
        if rank == 0:  # rank 1 skips this call: rank 0 waits for rows that never come
            t0 = time.perf_counter()
            layer(x)
            torch.cuda.synchronize()
            elapsed = time.perf_counter() - t0
        status = device_status(clear=True)
        set_wait_limit_ns(2_000_000_000)
        dist.barrier()  # host-side: rank 1 learns here that the step failed; no kernel of it is in flight
        peers.close()   # the group's epochs now differ: it is torn down, not reused
        out = {"good": good, "timed_out": bool(status & STATUS_WAIT_TIMEOUT), "status": status, "elapsed": elapsed}
    finally:
        torch.save(out, f"{result_path}.{rank}")
        dist.destroy_process_group()


def test_lost_peer_makes_the_fused_allreduce_time_out(tmp_path):
    """Rank 1 skips one fused GEMV + all-reduce call: rank 0's wait for its
    rows runs out (100 ms limit), the kernel returns with the timed-out bit,
    rank 1 sees nothing wrong on the device, and the group is torn down."""
    import torch.multiprocessing as mp

    _need(2)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_lost_peer_main, args=(2, _free_port(), str(tmp_path / "lost")), nprocs=2, join=True)
    r0, r1 = (torch.load(tmp_path / f"lost.{r}") for r in range(2))
    assert r0["good"] <= TOLERANCE and r1["good"] <= TOLERANCE
    assert r0["timed_out"], r0
    assert r0["elapsed"] < 10.0, r0
    assert r1["status"] == 0, r1


def _chain_allreduce_main(rank, world, port, result_path):
    import datetime

    import torch.distributed as dist

    from se12_b200.chain import Se12Chain
    from se12_b200.device import device_status
    from se12_b200.format import make_tensor
    from se12_b200.peers import PeerGroup
    from se12_b200.sharding import col_range, shard_matrix

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    out = {}
    try:
        mats = {}
        for name, rows, cols, seed in (("a", 1040, 4608, 8), ("b", 2304, 2048, 9)):
            bits, _, _ = cases.synthetic_weights(rows, cols, seed=seed, outlier_rate=2e-3, outlier_scale=256.0)
            s = oracle.encode(np.asarray(bits, dtype=np.uint16), rows, cols)
            t = make_tensor(s.rows, s.cols, s.codebook, s.sm, s.ec, s.esc, s.fallback_bitmap, s.fallback_raw)
            mats[name] = (bits, rows, cols, shard_matrix(t, "cols", world, rank, device=f"cuda:{rank}").matrix)
        peers = PeerGroup(rows_cap=2304)
        batch = 2
        chain = Se12Chain(batch)
        entries = []
        for n, name in enumerate(("a", "b", "a")):
            bits, rows, cols, m = mats[name]
            xb = oracle.bf16_round(np.random.default_rng(10 + n).normal(size=(batch, cols)).astype(np.float32))
            c0, c1 = col_range(cols, world, rank)
            x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()[:, c0:c1].contiguous()
            y = torch.full((batch, rows), float("nan"), device="cuda")
            chain.add(m, x, y, peers=peers)
            entries.append((bits, rows, cols, xb, y))
        errs, same = [], []
        for _ in range(2):  # two launches: the epochs continue across them
            chain.run()
            torch.cuda.synchronize()
            for bits, rows, cols, xb, y in entries:
                y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
                errs.append(oracle.max_relative_error(y.cpu().numpy(), y64))
                everyone = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(everyone, y)
                same.append(all(torch.equal(everyone[0], e) for e in everyone))
        out = {"errs": errs, "same": same, "status": device_status()}
        del chain
        peers.close()
    finally:
        torch.save(out, f"{result_path}.{rank}")
        dist.destroy_process_group()


def test_chain_with_allreduced_ops(tmp_path):
    """A chain whose ops are column shards all-reduced over the peer group
    inside the persistent kernel: within 1e-3 of the fp64 oracle, the same
    bits on every rank, over two launches."""
    import torch.multiprocessing as mp

    _need(2)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_chain_allreduce_main, args=(2, _free_port(), str(tmp_path / "chain")), nprocs=2, join=True)
    for r in range(2):
        res = torch.load(tmp_path / f"chain.{r}")
        assert res["status"] == 0, res
        assert max(res["errs"]) <= TOLERANCE, res["errs"]
        assert all(res["same"]), res["same"]


def _allgather_main(rank, world, port, result_path):
    import datetime

    import torch.distributed as dist

    from se12_b200.device import DeviceSe12Matrix, device_status
    from se12_b200.peers import PeerGroup
    from se12_b200.sharding import row_range

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    out = {}
    try:
        rows, cols = 128 * world, 2304  # equal 16-row-multiple shards
        bits, _, _ = cases.synthetic_weights(rows, cols, seed=12, outlier_rate=2e-3, outlier_scale=256.0)
        r0, r1 = row_range(rows, world, rank)
        shard = np.asarray(bits, dtype=np.uint16).reshape(rows, cols)[r0:r1].reshape(-1)
        s = oracle.encode(shard, r1 - r0, cols)

        def up(a, dtype):
            return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(dtype)).cuda()

        m = DeviceSe12Matrix(s.rows, s.cols, s.codebook, up(s.sm, np.uint8), up(s.ec, np.uint8), up(s.esc, np.uint8),
                             up(s.fallback_bitmap, np.uint8), up(s.fallback_raw, np.int16))
        peers = PeerGroup(rows_cap=r1 - r0)
        errs, same = [], []
        for call, batch in enumerate((1, 3, 16, 2)):
            xb = oracle.bf16_round(np.random.default_rng(call).normal(size=(batch, cols)).astype(np.float32))
            x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
            y = peers.gemv_allgather(m, x, r0, rows)
            y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
            errs.append(oracle.max_relative_error(y.cpu().numpy(), y64))
            everyone = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(everyone, y)
            same.append(all(torch.equal(everyone[0], e) for e in everyone))
        # from a CUDA graph, two calls per replay
        xb = oracle.bf16_round(np.random.default_rng(99).normal(size=(4, cols)).astype(np.float32))
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
        y = torch.empty(4, rows, device="cuda")
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            peers.gemv_allgather(m, x, r0, rows, out=y)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            peers.gemv_allgather(m, x, r0, rows, out=y)
            peers.gemv_allgather(m, x, r0, rows, out=y)
        y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
        for _ in range(3):
            y.zero_()
            graph.replay()
            torch.cuda.synchronize()
            errs.append(oracle.max_relative_error(y.cpu().numpy(), y64))
        del graph
        torch.cuda.synchronize()
        out = {"errs": errs, "same": same, "status": device_status()}
        peers.close()
    finally:
        torch.save(out, f"{result_path}.{rank}")
        dist.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_fused_gemv_allgather_over_peer_memory(tmp_path, world):
    """Row shards whose GEMV and all-gather are one kernel: every rank holds
    the whole output, within 1e-3 of the fp64 oracle and with the same bits
    on every rank, over calls in a row and from a replayed CUDA graph."""
    import torch.multiprocessing as mp

    _need(world)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_allgather_main, args=(world, _free_port(), str(tmp_path / "ag")), nprocs=world, join=True)
    for r in range(world):
        res = torch.load(tmp_path / f"ag.{r}")
        assert res["status"] == 0, res
        assert max(res["errs"]) <= TOLERANCE, res["errs"]
        assert all(res["same"]), res["same"]
