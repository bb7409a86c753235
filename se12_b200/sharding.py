"""Tensor-parallel sharding of SE12 matrices (multi-GPU, one process per GPU).

Shards are cut from the packed streams, never re-encoded, so every shard
decodes to exactly the matching slice of the original matrix and keeps the
tensor-wide codebook:

* ``shard_rows`` (output-parallel): tile rows [r0, r1) of the 16x256 tile
  grid. In tile-major order those tiles are one contiguous run of the sm /
  ec / esc streams, and their fallback tiles one contiguous run of
  ``fallback_raw``.
* ``shard_cols`` (input-parallel): tile columns [c0, c1) of every tile row,
  i.e. K split at 256-column boundaries; the tiles are gathered row by row.

``ShardedLinear`` runs the local fused GEMV, then the collective that
completes the layer: an all-gather of the output slices (row shards) or an
all-reduce of the partial sums (column shards), through ``torch.distributed``
(NCCL on GPUs). ``megatron_plan`` pairs them as in a transformer block
(q/k/v/gate/up by rows, o/down by columns, the LM head by rows), which needs
one all-reduce per attention block and one per MLP block.
"""

from __future__ import annotations

import typing

import numpy as np
import torch

from .format import ESCAPE_BUDGET, TILE_COLS, TILE_ROWS, TILE_SIZE, Se12Tensor, as_tensor, make_tensor, tile_grid


def split_points(n: int, parts: int) -> list:
    """Boundaries of ``parts`` near-equal contiguous ranges of ``n`` items."""
    if parts < 1:
        raise ValueError("parts must be >= 1")
    return [(n * p) // parts for p in range(parts + 1)]


def _fallback_bits(t: Se12Tensor) -> np.ndarray:
    return np.unpackbits(t.fallback_bitmap, count=t.tile_count).astype(bool)


def _subset(t: Se12Tensor, tile_ids: np.ndarray, rows: int, cols: int) -> Se12Tensor:
    """The SE12 tensor made of the given tiles (in that order) of ``t``."""
    tiles = t.tile_count
    sm = t.sm.reshape(tiles, TILE_SIZE)[tile_ids].reshape(-1)
    ec = t.ec.reshape(tiles, TILE_SIZE // 2)[tile_ids].reshape(-1)
    esc = t.esc.reshape(tiles, ESCAPE_BUDGET)[tile_ids]
    fb = _fallback_bits(t)
    rank = np.cumsum(fb) - 1
    raw_tiles = t.fallback_raw.reshape(-1, TILE_SIZE)
    chosen = tile_ids[fb[tile_ids]]
    raw = raw_tiles[rank[chosen]].reshape(-1) if chosen.size else np.zeros(0, dtype=np.int16)
    bitmap = np.packbits(fb[tile_ids].astype(np.uint8))
    return make_tensor(rows, cols, t.codebook, sm, ec, esc, bitmap, raw)


def shard_rows(tensor, parts: int, rank: int) -> Se12Tensor:
    """Output-parallel shard ``rank`` of ``parts``: a contiguous range of
    whole tile rows (16 output rows each; the last shard keeps the padding
    rows of the final tile row)."""
    t = as_tensor(tensor)
    tr, tc = tile_grid(t.rows, t.cols)
    if parts > tr:
        raise ValueError(f"{parts} row shards of a matrix with {tr} tile rows")
    b = split_points(tr, parts)
    r0, r1 = b[rank], b[rank + 1]
    rows = min(r1 * TILE_ROWS, t.rows) - r0 * TILE_ROWS
    ids = np.arange(r0 * tc, r1 * tc)
    return _subset(t, ids, rows, t.cols)


def shard_cols(tensor, parts: int, rank: int) -> Se12Tensor:
    """Input-parallel shard ``rank`` of ``parts``: a contiguous range of
    whole tile columns (K split at 256-column boundaries; the last shard
    keeps the padding columns of the final tile column)."""
    t = as_tensor(tensor)
    tr, tc = tile_grid(t.rows, t.cols)
    if parts > tc:
        raise ValueError(f"{parts} column shards of a matrix with {tc} tile columns")
    b = split_points(tc, parts)
    c0, c1 = b[rank], b[rank + 1]
    cols = min(c1 * TILE_COLS, t.cols) - c0 * TILE_COLS
    ids = (np.arange(tr)[:, None] * tc + np.arange(c0, c1)[None, :]).reshape(-1)
    return _subset(t, ids, t.rows, cols)


def row_range(rows: int, parts: int, rank: int) -> tuple:
    """Output rows [start, stop) that row shard ``rank`` produces."""
    tr = -(-rows // TILE_ROWS)
    b = split_points(tr, parts)
    return b[rank] * TILE_ROWS, min(b[rank + 1] * TILE_ROWS, rows)


def col_range(cols: int, parts: int, rank: int) -> tuple:
    """Input columns [start, stop) that column shard ``rank`` consumes."""
    tc = -(-cols // TILE_COLS)
    b = split_points(tc, parts)
    return b[rank] * TILE_COLS, min(b[rank + 1] * TILE_COLS, cols)


class ShardedLinear(torch.nn.Module):
    """One rank's part of a tensor-parallel SE12 linear layer.

    ``kind`` is ``"rows"`` (this rank holds output rows ``row_range``; the
    full output is all-gathered) or ``"cols"`` (this rank holds input
    columns ``col_range``; the partial sums are all-reduced). ``local``
    computes this rank's product (by default the fused GEMV of ``matrix``:
    x [B, k_local] -> fp32 [B, n_local]). With ``peers`` (a
    ``peers.PeerGroup``), a ``"cols"`` layer runs the GEMV and its
    all-reduce as one kernel over peer memory instead of a GEMV followed by
    an NCCL all-reduce, and a ``"rows"`` layer its GEMV and all-gather (the
    group's ``rows_cap`` x world must reach the layer's rows).
    """

    def __init__(self, kind: str, rows: int, cols: int, world: int, rank: int, matrix=None,
                 local: typing.Callable | None = None, group=None, peers=None):
        super().__init__()
        if kind not in ("rows", "cols"):
            raise ValueError("kind must be 'rows' or 'cols'")
        self.kind, self.rows, self.cols, self.world, self.rank = kind, rows, cols, world, rank
        self.matrix = matrix
        self.local = local if local is not None else (lambda x: matrix.gemv(x))
        self.group = group
        self.peers = peers
        self.row_bounds = [row_range(rows, world, r) for r in range(world)]
        self.col_bounds = [col_range(cols, world, r) for r in range(world)]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        x2 = x.reshape(-1, x.shape[-1])
        if self.kind == "cols":
            c0, c1 = self.col_bounds[self.rank]
            if self.peers is not None and self.world > 1:
                y = self.peers.gemv_allreduce(self.matrix, x2[:, c0:c1].contiguous().to(torch.bfloat16))
                return y.reshape(*x.shape[:-1], self.rows)
            y = self.local(x2[:, c0:c1].contiguous()).float()
            if self.world > 1:
                dist.all_reduce(y, group=self.group)
            return y.reshape(*x.shape[:-1], self.rows)
        if self.peers is not None and self.world > 1:
            r0, _ = self.row_bounds[self.rank]
            y = self.peers.gemv_allgather(self.matrix, x2.to(torch.bfloat16), r0, self.rows)
            return y.reshape(*x.shape[:-1], self.rows)
        y = self.local(x2).float()
        if self.world > 1:
            # shards differ by at most one tile row: gather equal-size
            # (padded) slices, then drop the padding
            sizes = [b - a for a, b in self.row_bounds]
            width = max(sizes)
            if y.shape[1] != width:
                y = torch.nn.functional.pad(y, (0, width - y.shape[1]))
            parts = [torch.empty(x2.shape[0], width, dtype=y.dtype, device=y.device) for _ in range(self.world)]
            dist.all_gather(parts, y.contiguous(), group=self.group)
            y = torch.cat([part[:, :n] for part, n in zip(parts, sizes)], dim=1)
        return y.reshape(*x.shape[:-1], self.rows)


def megatron_plan(name: str) -> str:
    """Shard kind of a decoder projection by its module name: attention
    output and MLP down projections by input columns (followed by an
    all-reduce), everything else by output rows."""
    leaf = name.rsplit(".", 1)[-1]
    return "cols" if leaf in ("o_proj", "down_proj", "out_proj", "wo", "w2") else "rows"


def shard_matrix(tensor, kind: str, world: int, rank: int, device="cuda", group=None, peers=None) -> ShardedLinear:
    """Uploads rank ``rank``'s shard of an SE12 tensor and wraps it (``peers``:
    fused GEMV + all-reduce for column shards)."""
    from .device import DeviceSe12Matrix

    t = as_tensor(tensor)
    part = shard_rows(t, world, rank) if kind == "rows" else shard_cols(t, world, rank)
    return ShardedLinear(kind, t.rows, t.cols, world, rank, DeviceSe12Matrix.from_tensor(part, device), group=group,
                         peers=peers)


__all__ = [
    "ShardedLinear",
    "col_range",
    "megatron_plan",
    "row_range",
    "shard_cols",
    "shard_matrix",
    "shard_rows",
    "split_points",
]
