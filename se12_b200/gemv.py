"""GEMV entry point with the reference adapter's interface
(src/lws/adapters/cuda/gemv.py:143-226), backed by libse12_b200.

``Se12MatVecKernel(compiler, target, tensor, sm_count, extra_decode_ops=0)``
and ``RawBf16MatVecKernel(compiler, target, weights, sm_count)`` keep the
reference constructors; ``compiler`` and ``target`` are accepted and ignored
(there is one ahead-of-time sm_100a build, no NVRTC), ``sm_count`` is read
from the device. ``multiply(activations, launch=None)`` returns fp32
[B, N] like the reference (the ``launch`` override is ignored: launch
geometry comes from the library's fixed per-shape table).
"""

from __future__ import annotations

import torch

from .device import DeviceSe12Matrix, bf16_gemv, gemv_call
from .format import fallback_offsets, tile_grid

__all__ = ["Se12MatVecKernel", "RawBf16MatVecKernel", "fallback_offsets", "tile_grid"]


def _device_of(activations_or_none=None) -> torch.device:
    return torch.device("cuda", torch.cuda.current_device())


class Se12MatVecKernel:
    """Bound to one SE12-encoded matrix (reference gemv.py:180-226)."""

    def __init__(self, compiler=None, target=None, tensor=None, sm_count=None, extra_decode_ops: int = 0, device=None):
        if tensor is None:
            raise ValueError("Se12MatVecKernel needs an SE12 tensor")
        if extra_decode_ops:
            raise ValueError("extra_decode_ops (the reference's decode-cost experiment) is not supported")
        dev = torch.device(device) if device is not None else _device_of()
        self.matrix = tensor if isinstance(tensor, DeviceSe12Matrix) else DeviceSe12Matrix.from_tensor(tensor, dev)
        self.output_rows = self.matrix.rows
        self.k = self.matrix.cols

    def multiply(self, activations: torch.Tensor, launch=None) -> torch.Tensor:
        x = activations if activations.is_cuda else activations.to(self.matrix.device)
        return gemv_call(self.matrix, x)


class RawBf16MatVecKernel:
    """Dense BF16 baseline bound to one [N, K] matrix (reference gemv.py:143-172)."""

    def __init__(self, compiler=None, target=None, weights: torch.Tensor = None, sm_count=None, device=None):
        if weights is None:
            raise ValueError("RawBf16MatVecKernel needs a BF16 weight matrix")
        dev = torch.device(device) if device is not None else _device_of()
        w = weights.to(dev)
        if w.dtype == torch.int16:
            w = w.view(torch.bfloat16)
        self.weights = w.contiguous()
        self.output_rows, self.k = self.weights.shape

    def multiply(self, activations: torch.Tensor, launch=None) -> torch.Tensor:
        x = activations if activations.is_cuda else activations.to(self.weights.device)
        return bf16_gemv(self.weights, x)
