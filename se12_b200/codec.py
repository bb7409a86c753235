"""SE12 encode / decode with the reference codec's interface, run on the GPU.

``encode_tensor(weights, shape)`` and ``decode_tensor(tensor)`` keep the
signatures of src/lws/domain/se12/codec.py:111 and :144 and produce
byte-identical streams / bit-exact weights, but the work happens in the
encoder and decoder kernels of libse12_b200 (there is no CPU codec in this
package). ``encode_device`` packs a BF16 matrix that is already on the GPU
and returns a ``DeviceSe12Matrix`` without a host round trip.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .device import DeviceSe12Matrix, stream_handle
from .format import (
    CODEBOOK_SIZE,
    ESCAPE_BUDGET,
    TILE_SIZE,
    Bf16Weights,
    MatrixShape,
    Se12Tensor,
    as_tensor,
    byte_size,
    fallback_tile_count,
    tile_grid,
)

__all__ = [
    "encode_tensor",
    "decode_tensor",
    "encode_device",
    "codebook_from_counts",
    "byte_size",
    "fallback_tile_count",
]


def codebook_from_counts(counts) -> tuple:
    """The 15 most frequent exponents of a 256-bin histogram, ties to the larger
    exponent (src/lws/domain/se12/codebook.py:41-59), computed by the library."""
    c = np.ascontiguousarray(np.asarray(counts, dtype=np.uint32).reshape(256))
    out = (ctypes.c_uint8 * CODEBOOK_SIZE)()
    _lib.call("se12_codebook_from_counts", ctypes.c_void_p(c.ctypes.data), out)
    return tuple(int(v) for v in out)


def encode_device(weights: torch.Tensor) -> DeviceSe12Matrix:
    """Packs a device BF16 [rows, cols] matrix into SE12 on the GPU."""
    if weights.dtype != torch.bfloat16 or weights.dim() != 2 or not weights.is_cuda:
        raise ValueError("encode_device needs a 2-D BF16 CUDA tensor")
    w = weights if weights.stride(1) == 1 else weights.contiguous()
    rows, cols = w.shape
    dev = w.device
    tr, tc = tile_grid(rows, cols)
    tiles = tr * tc
    stream = ctypes.c_void_p(stream_handle(dev))
    with torch.cuda.device(dev):
        counts = torch.empty(256, dtype=torch.int32, device=dev)
        _lib.call("se12_encode_histogram", ctypes.c_void_p(w.data_ptr()), rows, cols, w.stride(0),
                  ctypes.c_void_p(counts.data_ptr()), stream)
        codebook = codebook_from_counts(counts.cpu().numpy().view(np.uint32))
        book = (ctypes.c_uint8 * CODEBOOK_SIZE)(*codebook)
        sm = torch.empty(tiles * TILE_SIZE, dtype=torch.uint8, device=dev)
        ec = torch.empty(tiles * TILE_SIZE // 2, dtype=torch.uint8, device=dev)
        esc = torch.empty(tiles * ESCAPE_BUDGET, dtype=torch.uint8, device=dev)
        flags = torch.empty(tiles, dtype=torch.uint8, device=dev)
        _lib.call("se12_encode_tiles", ctypes.c_void_p(w.data_ptr()), rows, cols, w.stride(0), book,
                  ctypes.c_void_p(sm.data_ptr()), ctypes.c_void_p(ec.data_ptr()), ctypes.c_void_p(esc.data_ptr()),
                  ctypes.c_void_p(flags.data_ptr()), stream)
        bitmap = torch.empty((tiles + 7) // 8, dtype=torch.uint8, device=dev)
        findex = torch.empty(tiles, dtype=torch.int32, device=dev)
        fcount = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.call("se12_encode_bitmap", ctypes.c_void_p(flags.data_ptr()), tiles, ctypes.c_void_p(bitmap.data_ptr()),
                  ctypes.c_void_p(findex.data_ptr()), ctypes.c_void_p(fcount.data_ptr()), stream)
        nfall = int(fcount.item())
        raw = torch.empty(max(nfall, 0) * TILE_SIZE, dtype=torch.int16, device=dev)
        if nfall:
            _lib.call("se12_encode_raw", ctypes.c_void_p(w.data_ptr()), rows, cols, w.stride(0),
                      ctypes.c_void_p(findex.data_ptr()), ctypes.c_void_p(raw.data_ptr()), stream)
    return DeviceSe12Matrix(rows, cols, codebook, sm, ec, esc, bitmap, raw)


def _bits_of(weights) -> np.ndarray:
    pattern = weights.bit_pattern if hasattr(weights, "bit_pattern") else np.asarray(weights)
    pattern = np.ascontiguousarray(pattern)
    if pattern.dtype == np.uint16:
        pattern = pattern.view(np.int16)
    if pattern.dtype != np.int16:
        raise ValueError("weights must be an int16 (or uint16) BF16 bit pattern")
    return pattern.reshape(-1)


def encode_tensor(weights, shape, device="cuda") -> Se12Tensor:
    """SE12 encode of a BF16 bit pattern (codec.py:111-141), on the GPU.
    ``weights``: Bf16Weights (or an int16/uint16 array); ``shape``: object with
    .rows/.cols or a (rows, cols) tuple. Returns host streams."""
    rows, cols = (shape.rows, shape.cols) if hasattr(shape, "rows") else tuple(shape)
    bits = _bits_of(weights)
    if bits.size != rows * cols:
        raise ValueError(f"{bits.size} weights do not fit shape {rows}x{cols}")
    w = torch.from_numpy(bits.copy()).view(torch.bfloat16).reshape(rows, cols).to(device)
    return encode_device(w).to_tensor()


def decode_tensor(tensor, device="cuda") -> Bf16Weights:
    """Exact BF16 bits of an Se12Tensor (codec.py:144-186), decoded on the GPU."""
    m = DeviceSe12Matrix.from_tensor(as_tensor(tensor), device=device)
    out = m.decode()
    return Bf16Weights(bit_pattern=out.view(torch.int16).reshape(-1).cpu().numpy())


def round_trip_shape(rows: int, cols: int) -> MatrixShape:
    return MatrixShape(rows, cols)
