"""GPU weight decoder with the reference adapter's interface
(src/lws/adapters/cuda/se12_decoder.py:45-76, port
src/lws/application/ports/gpu/weight_decoder.py:26-33), backed by the
decode kernels of libse12_b200.

``decode_rows`` decodes only the requested rows (the reference decodes the
whole tensor and slices it).
"""

from __future__ import annotations

import dataclasses

import torch

from .device import DeviceSe12Matrix
from .format import Bf16Weights, as_tensor


@dataclasses.dataclass(frozen=True)
class RowIndices:
    """Matrix rows to decode, in request order (weight_decoder.py:19-23)."""

    values: tuple


class CudaSe12WeightDecoder:
    def __init__(self, compiler=None, target=None, device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())

    def _matrix(self, tensor) -> DeviceSe12Matrix:
        if isinstance(tensor, DeviceSe12Matrix):
            return tensor
        return DeviceSe12Matrix.from_tensor(as_tensor(tensor), self.device)

    def decode(self, tensor) -> Bf16Weights:
        out = self._matrix(tensor).decode()
        return Bf16Weights(bit_pattern=out.view(torch.int16).reshape(-1).cpu().numpy())

    def decode_to_device(self, tensor) -> torch.Tensor:
        """The decoded BF16 matrix, resident on the GPU."""
        return self._matrix(tensor).decode()

    def decode_rows(self, tensor, rows) -> Bf16Weights:
        values = rows.values if hasattr(rows, "values") else tuple(rows)
        out = self._matrix(tensor).decode_rows(list(values))
        return Bf16Weights(bit_pattern=out.view(torch.int16).reshape(-1).cpu().numpy())
