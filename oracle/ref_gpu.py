"""The reference's own GPU kernel (lws_gemv_se12), driven from Python.

TEST AND COMPARISON INFRASTRUCTURE, not the product: oracle/_ref/
libref_kernels.so holds the reference's kernels compiled unchanged for
sm_100a (oracle/build_ref.py). The GPU parity tests run the kernel here
against the oracle, and bench.py's reference arm times it beside the
reference's CPU path. Nothing in se12_b200/ imports this module.

What the reference's host code does before a launch is restated here:
* ``fallback_offsets``: each tile's rank among fallback tiles
  (src/lws/adapters/cuda/gemv.py:47-57);
* ``row_escape_offset``: per output row and tile column, the escapes in the
  earlier rows of that row's tile (gemv.py:60-77);
* ``default_launch``: threads per block from {256, 128, 64, 32}, the
  largest that still gives 4 blocks per SM, one warp per (row, batch)
  (src/lws/domain/launch/heuristic.py:46-51).
The tables are computed with torch on the matrix's device; the numpy
restatement in se12_oracle is pinned to the reference's own helpers by
tests/golden/golden_ref_tables.json.
"""

from __future__ import annotations

import ctypes
import pathlib

import torch

LIBRARY = pathlib.Path(__file__).resolve().parent / "_ref" / "libref_kernels.so"
THREADS_PER_BLOCK_CANDIDATES = (256, 128, 64, 32)
TARGET_BLOCKS_PER_SM = 4

_LIB = None


def available() -> bool:
    return LIBRARY.exists()


def load() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIBRARY.exists():
            raise RuntimeError(f"{LIBRARY} is missing: build it with python oracle/build_ref.py <reference-tree>")
        lib = ctypes.CDLL(str(LIBRARY))
        vp, i = ctypes.c_void_p, ctypes.c_int
        lib.ref_gemv_se12.argtypes = [vp] * 10 + [i] * 5 + [vp]
        lib.ref_gemv_se12.restype = i
        _LIB = lib
    return _LIB


def default_launch(sm_count: int, rows: int, batch: int) -> tuple:
    """(blocks, threads per block) of the reference's heuristic."""
    warps = rows * batch
    target = sm_count * TARGET_BLOCKS_PER_SM
    fitting = [t for t in THREADS_PER_BLOCK_CANDIDATES if -(-warps // (t // 32)) >= target]
    threads = max(fitting) if fitting else 32
    return -(-warps // (threads // 32)), threads


def fallback_offsets(bitmap: torch.Tensor, tiles: int) -> torch.Tensor:
    """int32 [tiles]: cumulative count of fallback tiles up to each tile,
    minus one (bit 7 - i % 8 of byte i / 8, MSB first)."""
    shifts = torch.arange(7, -1, -1, device=bitmap.device, dtype=torch.int32)
    bits = ((bitmap.to(torch.int32)[:, None] >> shifts) & 1).reshape(-1)[:tiles]
    return (torch.cumsum(bits, 0) - 1).to(torch.int32)


def row_escape_offset(ec: torch.Tensor, tile_rows: int, tile_cols: int) -> torch.Tensor:
    """int32 [16 tile_rows, tile_cols]: for output row n and tile column kt,
    the escapes (code 15) in rows 0 .. n % 16 - 1 of tile (n / 16, kt)."""
    tiles = tile_rows * tile_cols
    packed = ec[: tiles * 2048].reshape(tiles, 16, 128).to(torch.int32)
    escapes = ((packed & 0xF) == 15).to(torch.int32) + ((packed >> 4) == 15).to(torch.int32)  # both nibbles of a byte
    per_row = escapes.sum(dim=2)                                  # [tiles, 16]
    exclusive = torch.cumsum(per_row, dim=1) - per_row            # [tiles, 16]
    return exclusive.reshape(tile_rows, tile_cols, 16).permute(0, 2, 1).reshape(tile_rows * 16, tile_cols).to(
        torch.int32).contiguous()


class RefSe12Gemv:
    """One SE12 matrix (a DeviceSe12Matrix-like object with sm, ec, esc,
    codebook, fallback_bitmap, fallback_raw, rows, cols, tile_rows,
    tile_cols, tiles) and the side tables the reference kernel reads."""

    def __init__(self, m, sm_count: int):
        if m.cols % 256:
            raise ValueError("the reference kernel needs cols % 256 == 0 (gemv_se12.cu:17-21)")
        dev = m.sm.device
        self.m = m
        self.sm_count = sm_count
        self.codebook = torch.tensor(list(m.codebook), dtype=torch.uint8, device=dev)
        self.fallback_offsets = fallback_offsets(m.fallback_bitmap, m.tiles)
        self.row_escape_offset = row_escape_offset(m.ec, m.tile_rows, m.tile_cols)
        # 64 spare bytes behind esc: the kernel reads escape slots by rank
        self.esc = torch.zeros(m.esc.numel() + 64, dtype=torch.uint8, device=dev)
        self.esc[: m.esc.numel()].copy_(m.esc)
        raw = m.fallback_raw
        self.raw = raw if raw.numel() else torch.zeros(4096, dtype=torch.int16, device=dev)

    def launch(self, x: torch.Tensor, y: torch.Tensor, stream: int) -> None:
        """y[B, rows] = x[B, cols] (fp32, contiguous) times the matrix."""
        batch = x.shape[0]
        blocks, threads = default_launch(self.sm_count, self.m.rows, batch)
        m = self.m
        p = ctypes.c_void_p
        rc = load().ref_gemv_se12(p(m.sm.data_ptr()), p(m.ec.data_ptr()), p(self.esc.data_ptr()),
                                  p(self.codebook.data_ptr()), p(m.fallback_bitmap.data_ptr()),
                                  p(self.fallback_offsets.data_ptr()), p(self.raw.data_ptr()),
                                  p(self.row_escape_offset.data_ptr()), p(x.data_ptr()), p(y.data_ptr()),
                                  m.rows, m.cols, batch, blocks, threads, p(stream))
        if rc != 0:
            raise RuntimeError(f"lws_gemv_se12 launch failed: CUDA error {rc}")
