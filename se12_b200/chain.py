"""Chains: a sequence of GEMVs run in order by one persistent launch.

``Se12Chain`` wraps the ``se12_chain_*`` C ABI. A decode step's projections
(q/k/v, o, gate/up, down of every layer, then the LM head) are added in
order with their input and output buffers; ``run()`` launches the whole
sequence as one kernel on the current stream. Op j reads its x only after
op j - 1 has finished on every CTA, so each op may take its input from the
previous op's output; the weights of the next op stream in meanwhile. This
is the stacked mode of the reference's microbenchmark design
(.spec/features/fused-decode-gemv/design.md:155-165) taken into one kernel.

The chain keeps references to every tensor it was given (matrices, their
tile records, x and y): the buffers must not be replaced, only refilled.
"""

from __future__ import annotations

import ctypes
import weakref

import torch

from . import _lib
from .device import DeviceSe12Matrix, stream_handle


def _check_x(x: torch.Tensor, cols: int, batch: int) -> None:
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be a BF16 [batch, ldx] tensor with unit column stride")
    if x.shape[0] != batch or x.shape[1] < cols or x.stride(0) % 8 or x.data_ptr() % 16:
        raise ValueError(f"x must be [{batch}, >= {cols}] with 16-byte aligned rows (ldx % 8 == 0)")


def _check_y(y: torch.Tensor, rows: int, batch: int) -> None:
    if y.dtype != torch.float32 or y.dim() != 2 or y.stride(1) != 1 or y.shape[0] != batch or y.shape[1] < rows:
        raise ValueError(f"y must be an fp32 [{batch}, >= {rows}] tensor with unit column stride")


class Se12Chain:
    """GEMVs of one batch size, run in order by one launch (``dense``: a
    chain of dense BF16 GEMVs, the comparison baseline)."""

    def __init__(self, batch: int, device: torch.device | str = "cuda", dense: bool = False):
        lib = _lib.load()
        self.device = torch.device(device)
        self.batch = int(batch)
        self.dense = bool(dense)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.se12_chain_create(self.batch, 1 if dense else 0, ctypes.byref(handle)), "se12_chain_create")
        self._handle = handle
        self._finalizer = weakref.finalize(self, lib.se12_chain_destroy, handle)
        self._keep: list = []
        self._descriptors = None
        self._workspace = None
        self.gemvs = 0

    def add(self, matrix: DeviceSe12Matrix, x: torch.Tensor, y: torch.Tensor, peers=None) -> None:
        """y[:, :rows] = x[:, :cols] . W^T; with ``peers`` (a PeerGroup used
        by this chain only or with the same call order on every rank), the
        rows are summed over the group's ranks (column-sharded layer)."""
        if self.dense:
            raise ValueError("a dense chain takes dense GEMVs (add_dense)")
        self._check_open()
        _check_x(x, matrix.cols, self.batch)
        _check_y(y, matrix.rows, self.batch)
        rec = matrix.records
        args = (self._handle, matrix.handle, ctypes.c_void_p(rec.data_ptr()), ctypes.c_void_p(x.data_ptr()), x.stride(0),
                ctypes.c_void_p(y.data_ptr()), y.stride(0))
        if peers is None:
            _lib.call("se12_chain_add_gemv", *args)
        else:
            _lib.call("se12_chain_add_gemv_allreduce", *args, ctypes.byref(peers.struct))
        self._keep.extend([matrix, rec, x, y] + ([peers] if peers is not None else []))
        self.gemvs += 1

    def add_dense(self, weights: torch.Tensor, x: torch.Tensor, y: torch.Tensor) -> None:
        if not self.dense:
            raise ValueError("an SE12 chain takes SE12 GEMVs (add)")
        self._check_open()
        if weights.dtype != torch.bfloat16 or weights.dim() != 2 or weights.stride(1) != 1:
            raise ValueError("weights must be a BF16 [rows, cols] matrix with unit column stride")
        rows, cols = weights.shape
        _check_x(x, cols, self.batch)
        _check_y(y, rows, self.batch)
        _lib.call("se12_chain_add_dense", self._handle, ctypes.c_void_p(weights.data_ptr()), rows, cols, weights.stride(0),
                  ctypes.c_void_p(x.data_ptr()), x.stride(0), ctypes.c_void_p(y.data_ptr()), y.stride(0))
        self._keep.extend([weights, x, y])
        self.gemvs += 1

    def _check_open(self):
        if self._descriptors is not None:
            raise RuntimeError("the chain was uploaded: build a new chain to add GEMVs")

    @property
    def ops(self) -> int:
        """Ops after column splits (a GEMV whose x does not fit shared memory
        at this batch becomes several)."""
        return _lib.load().se12_chain_ops(self._handle)

    def info(self) -> dict:
        grid, consumers, smem, ops = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _lib.call("se12_chain_info", self._handle, ctypes.byref(grid), ctypes.byref(consumers), ctypes.byref(smem),
                  ctypes.byref(ops))
        return {"grid": grid.value, "consumer_warps": consumers.value, "threads": 32 * (consumers.value + 1),
                "smem_bytes": smem.value, "ops": ops.value, "gemvs": self.gemvs}

    def upload(self) -> None:
        """Copies the op descriptors to the device and zeroes the workspace
        (on the current stream)."""
        lib = _lib.load()
        nd = lib.se12_chain_descriptor_bytes(self._handle)
        nw = lib.se12_chain_workspace_bytes(self._handle)
        self._descriptors = torch.empty(nd, dtype=torch.uint8, device=self.device)
        self._workspace = torch.empty(nw, dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("se12_chain_upload", self._handle, ctypes.c_void_p(self._descriptors.data_ptr()),
                      ctypes.c_void_p(self._workspace.data_ptr()), nw, ctypes.c_void_p(stream_handle(self.device)))

    def run(self) -> None:
        """One launch of the whole chain on the current stream."""
        if self._descriptors is None:
            self.upload()
        with torch.cuda.device(self.device):
            _lib.call("se12_chain_run", self._handle, ctypes.c_void_p(stream_handle(self.device)))

    def reset(self) -> None:
        """Zeroes the workspace (after a kernel reported a timed-out wait)."""
        with torch.cuda.device(self.device):
            _lib.call("se12_chain_reset", self._handle, ctypes.c_void_p(stream_handle(self.device)))


__all__ = ["Se12Chain"]
