"""Peer groups for the fused GEMV + all-reduce (``se12_gemv_allreduce``).

Tensor parallelism with the input columns sharded (attention output and MLP
down projections) needs, after each rank's GEMV of its column shard, the sum
of all ranks' outputs on every rank. ``PeerGroup`` sets up what the fused
kernel needs for that across the ranks of a ``torch.distributed`` group,
one GPU per rank on one node: a receive buffer per rank (values tagged
with the call's epoch), mapped into every other rank's address space with
CUDA IPC
(``se12_ipc_handle`` / ``se12_ipc_open``: plain peer memory over NVLink, no
multicast object), and a per-rank call counter.
``gemv_allreduce`` then runs one kernel per call: no NCCL on this path.

Every rank must make the same calls on a group, in the same order, on one
stream per rank (what a tensor-parallel decode step does anyway).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .device import MAX_BATCH, WORKSPACES, DeviceSe12Matrix, _aligned_bf16, stream_handle

MAX_PEERS = 8


class PeerGroup:
    """Buffers of ``se12_gemv_allreduce`` for matrices of up to ``rows_cap``
    rows, shared by the ranks of ``group`` (collective: every rank builds
    its ``PeerGroup`` at the same point)."""

    def __init__(self, rows_cap: int, group=None, device: torch.device | str | None = None):
        import torch.distributed as dist

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= MAX_PEERS:
            raise ValueError(f"a peer group has 2..{MAX_PEERS} ranks, got {self.world}")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.rows_cap = int(rows_cap)
        lib = _lib.load()
        recv_bytes = lib.se12_peer_recv_bytes(self.world, self.rows_cap)
        # one buffer per rank, mapped once into every other rank
        self.buffer = torch.zeros(recv_bytes, dtype=torch.uint8, device=self.device)
        self.epoch = torch.zeros(4, dtype=torch.int32, device=self.device)  # this rank's call counter (not shared)
        torch.cuda.synchronize(self.device)
        handle = (ctypes.c_uint8 * 64)()
        offset = ctypes.c_uint64(0)
        with torch.cuda.device(self.device):
            _lib.call("se12_ipc_handle", ctypes.c_void_p(self.buffer.data_ptr()), handle, ctypes.byref(offset))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (bytes(handle), offset.value), group=group)
        self._mappings = []
        bases = []
        with torch.cuda.device(self.device):
            for r, (h, off) in enumerate(everyone):
                if r == self.rank:
                    bases.append(self.buffer.data_ptr())
                    continue
                ptr, mapping = ctypes.c_void_p(), ctypes.c_void_p()
                _lib.call("se12_ipc_open", (ctypes.c_uint8 * 64).from_buffer_copy(h), off, ctypes.byref(ptr), ctypes.byref(mapping))
                self._mappings.append(mapping.value)
                bases.append(ptr.value)
        self.struct = _lib.Se12PeerGroupStruct()
        self.struct.world, self.struct.rank, self.struct.rows_cap = self.world, self.rank, self.rows_cap
        for r in range(self.world):
            self.struct.recv[r] = bases[r]
        self.struct.epoch = self.epoch.data_ptr()
        self._group = group
        dist.barrier(group=group)

    def close(self) -> None:
        """Unmaps the other ranks' buffers (collective: every rank closes,
        after its last call on the group has finished)."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self._group)
        with torch.cuda.device(self.device):
            for mapping in self._mappings:
                _lib.call("se12_ipc_close", ctypes.c_void_p(mapping))
        self._mappings = []

    def gemv_allreduce(self, m: DeviceSe12Matrix, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """y = sum over ranks of this rank's ``m`` (its column shard) times
        ``x`` (BF16 [B, m.cols]); fp32 [B, m.rows], the same bits on every
        rank. Batches above 16 run as chunks of 16 (each chunk is a call)."""
        if x.dtype != torch.bfloat16:
            raise TypeError("activations must be bfloat16")
        if m.rows > self.rows_cap:
            raise ValueError(f"matrix has {m.rows} rows, the group holds {self.rows_cap}")
        squeeze = x.dim() == 1
        x2 = x.reshape(1, -1) if squeeze else x
        batch = x2.shape[0]
        if out is None:
            out = torch.empty(batch, m.rows, dtype=torch.float32, device=x.device)
        stream = stream_handle(x.device)
        lib = _lib.load()
        with torch.cuda.device(x.device):
            for b0 in range(0, batch, MAX_BATCH):
                xb = _aligned_bf16(x2[b0:b0 + MAX_BATCH], m.cols)
                yb = out[b0:b0 + MAX_BATCH]
                need = lib.se12_gemv_workspace_bytes(m.handle, MAX_BATCH)
                ws = WORKSPACES.get(x.device, stream, need)
                _lib.call("se12_gemv_allreduce", m.handle, ctypes.c_void_p(xb.data_ptr()), xb.shape[0], xb.stride(0),
                          ctypes.c_void_p(yb.data_ptr()), yb.stride(0), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                          ctypes.byref(self.struct), ctypes.c_void_p(stream))
        return out.reshape(-1) if squeeze else out

    def gemv_allgather(self, m: DeviceSe12Matrix, x: torch.Tensor, row0: int, rows_full: int,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """The whole rows_full-row output on every rank: this rank's ``m``
        holds rows row0 .. row0 + m.rows - 1 of it, times ``x`` (BF16 [B,
        m.cols]); fp32 [B, rows_full], the same bits on every rank. Batches
        above 16 run as chunks of 16 (each chunk is a call)."""
        if x.dtype != torch.bfloat16:
            raise TypeError("activations must be bfloat16")
        if rows_full > self.world * self.rows_cap:
            raise ValueError(f"{rows_full} gathered rows, the group holds {self.world} x {self.rows_cap}")
        squeeze = x.dim() == 1
        x2 = x.reshape(1, -1) if squeeze else x
        batch = x2.shape[0]
        if out is None:
            out = torch.empty(batch, rows_full, dtype=torch.float32, device=x.device)
        stream = stream_handle(x.device)
        lib = _lib.load()
        with torch.cuda.device(x.device):
            for b0 in range(0, batch, MAX_BATCH):
                xb = _aligned_bf16(x2[b0:b0 + MAX_BATCH], m.cols)
                yb = out[b0:b0 + MAX_BATCH]
                need = lib.se12_gemv_workspace_bytes(m.handle, MAX_BATCH)
                ws = WORKSPACES.get(x.device, stream, need)
                _lib.call("se12_gemv_allgather", m.handle, ctypes.c_void_p(xb.data_ptr()), xb.shape[0], xb.stride(0),
                          ctypes.c_void_p(yb.data_ptr()), yb.stride(0), int(row0), int(rows_full),
                          ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.byref(self.struct), ctypes.c_void_p(stream))
        return out.reshape(-1) if squeeze else out


__all__ = ["MAX_PEERS", "PeerGroup"]
