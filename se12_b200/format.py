"""SE12 tensor value types with the reference's public shape.

Code written against ``lws`` reads an encoded tensor as
``tensor.streams.primary.sm.value``, ``tensor.metadata.codebook.exponents``
and so on (src/lws/domain/se12/codec.py:33-107, tile.py:27-55,
codebook.py:19-30, weights.py:22-37). These classes keep those attribute
paths, so a ``Se12Tensor`` built by either package works with the other's
consumers; ``as_tensor`` also accepts the reference's own objects by duck
typing. Host arrays only: no computation happens here.
"""

from __future__ import annotations

import dataclasses

import numpy as np

TILE_ROWS = 16
TILE_COLS = 256
TILE_SIZE = TILE_ROWS * TILE_COLS
ESCAPE_BUDGET = 16
CODEBOOK_SIZE = 15
ESCAPE_CODE = 15
FORMAT_NAME = "SE12"
CURRENT_FORMAT_VERSION = 1
SUPPORTED_FORMAT_VERSIONS = (1,)


class UnsupportedFormatVersionError(ValueError):
    """A packed file declares a format version this codec does not know
    (the reference's lws.domain.se12.container.UnsupportedFormatVersionError)."""


@dataclasses.dataclass(frozen=True)
class FormatVersion:
    value: int


def validate_format_version(found: FormatVersion) -> None:
    """Refuses an unknown version, naming the found and supported ones
    (src/lws/domain/se12/container.py:21-27)."""
    if found.value in SUPPORTED_FORMAT_VERSIONS:
        return
    supported = ", ".join(str(v) for v in SUPPORTED_FORMAT_VERSIONS)
    raise UnsupportedFormatVersionError(f"found format version {found.value}, supported: {supported}")


@dataclasses.dataclass(frozen=True)
class Bf16Weights:
    """Flat int16 bit pattern of a BF16 tensor (weights.py:22-37)."""

    bit_pattern: np.ndarray

    def __post_init__(self):
        if self.bit_pattern.dtype != np.int16:
            raise ValueError("Bf16Weights requires an int16 bit-pattern view")
        if self.bit_pattern.ndim != 1:
            raise ValueError("Bf16Weights requires a flattened 1-D array")


@dataclasses.dataclass(frozen=True)
class MatrixShape:
    rows: int
    cols: int


@dataclasses.dataclass(frozen=True)
class TileShape:
    rows: int
    cols: int


@dataclasses.dataclass(frozen=True)
class EscapeBudget:
    value: int


@dataclasses.dataclass(frozen=True)
class Codebook:
    exponents: tuple

    def __post_init__(self):
        if len(self.exponents) != CODEBOOK_SIZE:
            raise ValueError(f"Codebook needs exactly {CODEBOOK_SIZE} entries, got {len(self.exponents)}")


@dataclasses.dataclass(frozen=True)
class Stream:
    """One stream array (the reference wraps each in its own `.value` class)."""

    value: np.ndarray


@dataclasses.dataclass(frozen=True)
class PrimaryStreams:
    sm: Stream
    ec: Stream


@dataclasses.dataclass(frozen=True)
class FallbackData:
    bitmap: Stream
    raw: Stream


@dataclasses.dataclass(frozen=True)
class EscapeHandling:
    esc: Stream
    fallback: FallbackData


@dataclasses.dataclass(frozen=True)
class Se12Streams:
    primary: PrimaryStreams
    escape_handling: EscapeHandling


@dataclasses.dataclass(frozen=True)
class TilingParameters:
    tile_shape: TileShape
    escape_budget: EscapeBudget


@dataclasses.dataclass(frozen=True)
class Se12Geometry:
    shape: MatrixShape
    tiling: TilingParameters


@dataclasses.dataclass(frozen=True)
class Se12Metadata:
    codebook: Codebook
    geometry: Se12Geometry


@dataclasses.dataclass(frozen=True)
class Se12Tensor:
    """A fully encoded SE12 tensor (codec.py:103-107)."""

    streams: Se12Streams
    metadata: Se12Metadata

    # flat accessors -------------------------------------------------------
    @property
    def rows(self) -> int:
        return self.metadata.geometry.shape.rows

    @property
    def cols(self) -> int:
        return self.metadata.geometry.shape.cols

    @property
    def codebook(self) -> tuple:
        return tuple(self.metadata.codebook.exponents)

    @property
    def sm(self) -> np.ndarray:
        return self.streams.primary.sm.value

    @property
    def ec(self) -> np.ndarray:
        return self.streams.primary.ec.value

    @property
    def esc(self) -> np.ndarray:
        return self.streams.escape_handling.esc.value

    @property
    def fallback_bitmap(self) -> np.ndarray:
        return self.streams.escape_handling.fallback.bitmap.value

    @property
    def fallback_raw(self) -> np.ndarray:
        return self.streams.escape_handling.fallback.raw.value

    @property
    def tile_grid(self) -> tuple:
        return tile_grid(self.rows, self.cols)

    @property
    def tile_count(self) -> int:
        tr, tc = self.tile_grid
        return tr * tc


def tile_grid(rows: int, cols: int) -> tuple:
    """(tile rows, tile cols) of a padded matrix (src/lws/adapters/cuda/gemv.py:89-92)."""
    return -(-rows // TILE_ROWS), -(-cols // TILE_COLS)


def make_tensor(rows, cols, codebook, sm, ec, esc, fallback_bitmap, fallback_raw) -> Se12Tensor:
    tr, tc = tile_grid(rows, cols)
    return Se12Tensor(
        streams=Se12Streams(
            primary=PrimaryStreams(sm=Stream(np.asarray(sm, dtype=np.uint8)), ec=Stream(np.asarray(ec, dtype=np.uint8))),
            escape_handling=EscapeHandling(
                esc=Stream(np.asarray(esc, dtype=np.uint8).reshape(tr * tc, ESCAPE_BUDGET)),
                fallback=FallbackData(
                    bitmap=Stream(np.asarray(fallback_bitmap, dtype=np.uint8)),
                    raw=Stream(np.asarray(fallback_raw).view(np.int16) if np.asarray(fallback_raw).dtype != np.int16 else np.asarray(fallback_raw)),
                ),
            ),
        ),
        metadata=Se12Metadata(
            codebook=Codebook(tuple(int(v) for v in codebook)),
            geometry=Se12Geometry(
                shape=MatrixShape(int(rows), int(cols)),
                tiling=TilingParameters(TileShape(TILE_ROWS, TILE_COLS), EscapeBudget(ESCAPE_BUDGET)),
            ),
        ),
    )


def as_tensor(tensor) -> Se12Tensor:
    """Accepts this package's Se12Tensor or the reference's (duck-typed)."""
    if isinstance(tensor, Se12Tensor):
        return tensor
    streams, metadata = tensor.streams, tensor.metadata
    geometry = metadata.geometry
    tiling = geometry.tiling
    if (tiling.tile_shape.rows, tiling.tile_shape.cols, tiling.escape_budget.value) != (TILE_ROWS, TILE_COLS, ESCAPE_BUDGET):
        raise ValueError("only the 16x256 tile shape with an escape budget of 16 is supported")
    return make_tensor(
        geometry.shape.rows,
        geometry.shape.cols,
        metadata.codebook.exponents,
        streams.primary.sm.value,
        streams.primary.ec.value,
        streams.escape_handling.esc.value,
        streams.escape_handling.fallback.bitmap.value,
        streams.escape_handling.fallback.raw.value,
    )


def byte_size(tensor) -> int:
    """Every byte an SE12 tensor occupies: five streams + 15 codebook bytes
    (src/lws/domain/se12/summary.py:71-86)."""
    t = as_tensor(tensor)
    return int(t.sm.nbytes + t.ec.nbytes + t.esc.nbytes + t.fallback_bitmap.nbytes + t.fallback_raw.nbytes + CODEBOOK_SIZE)


def fallback_tile_count(tensor) -> int:
    t = as_tensor(tensor)
    return int(np.unpackbits(t.fallback_bitmap, count=t.tile_count).sum())


def fallback_offsets(bitmap: np.ndarray, tile_count: int) -> np.ndarray:
    """Each tile's rank among fallback tiles (src/lws/adapters/cuda/gemv.py:47-53)."""
    bits = np.unpackbits(bitmap, count=tile_count)
    return (np.cumsum(bits.astype(np.int32)) - 1).astype(np.int32)
