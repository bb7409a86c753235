"""Packed SE12 models on disk: the safetensors container of ``lws.pack``.

Layout (src/lws/adapters/safetensors/packed_store.py:36-135): one output
file per input shard, same file name. Every eligible tensor (BF16 and 2-D,
src/lws/application/codec/pack_model.py:1-8, 112-131) is stored as its five
SE12 streams under ``<name>.se12.sm`` (u8 [T*4096]), ``.ec`` (u8 [T*2048]),
``.esc`` (u8 [T, 16]), ``.fallback_bitmap`` (u8 [ceil(T/8)]) and
``.fallback_raw`` (i16 [F*4096]); every other tensor is copied through under
its own name with its own dtype and shape. The file metadata holds one JSON
string under the key ``se12``: ``{"format": "SE12", "format_version": 1,
"tensors": {name: {...}}}`` with, per SE12 tensor, its shape, tile shape,
escape budget and codebook.

* ``pack_model`` is the packer (``python -m lws.pack <model_dir> <out_dir>``)
  with the encoding done on the GPU; its files are byte-identical to the
  reference's.
* ``read_packed`` / ``load_packed_tensors`` are the reader, which the
  reference has only as a test helper (tests/test_spec_pack.py:66-92).
"""

from __future__ import annotations

import dataclasses
import json
import pathlib
import typing

import numpy as np
import torch

from .format import (
    CURRENT_FORMAT_VERSION,
    ESCAPE_BUDGET,
    FORMAT_NAME,
    TILE_COLS,
    TILE_ROWS,
    FormatVersion,
    Se12Tensor,
    UnsupportedFormatVersionError,
    as_tensor,
    byte_size,
    make_tensor,
    validate_format_version,
)

SHARD_GLOB = "*.safetensors"
STREAM_SUFFIXES = ("sm", "ec", "esc", "fallback_bitmap", "fallback_raw")
METADATA_KEY = "se12"


def _safetensors():
    import safetensors
    import safetensors.torch

    return safetensors


# ---------------------------------------------------------------------- writing


def _se12_metadata(t: Se12Tensor) -> dict:
    # Same keys, order and values as the reference (packed_store.py:92-107).
    return {
        "eligible": True,
        "shape": [t.rows, t.cols],
        "dtype": "torch.bfloat16",
        "tile_rows": TILE_ROWS,
        "tile_cols": TILE_COLS,
        "escape_budget": ESCAPE_BUDGET,
        "codebook": list(t.codebook),
    }


def write_packed_shard(path: str | pathlib.Path, entries: typing.Iterable[tuple[str, object]]) -> None:
    """Writes one packed shard. ``entries``: (name, value) in the order the
    source shard lists its tensors; value is an SE12 tensor (this package's
    or the reference's) or a torch tensor copied through unchanged."""
    st = _safetensors()
    tensors: dict = {}
    metadata: dict = {}
    for name, value in entries:
        if isinstance(value, torch.Tensor):
            tensors[name] = value.detach().cpu().contiguous()
            metadata[name] = {"eligible": False, "shape": list(value.shape), "dtype": str(value.dtype)}
            continue
        t = as_tensor(value)
        tensors[f"{name}.se12.sm"] = torch.from_numpy(np.ascontiguousarray(t.sm).reshape(-1))
        tensors[f"{name}.se12.ec"] = torch.from_numpy(np.ascontiguousarray(t.ec).reshape(-1))
        tensors[f"{name}.se12.esc"] = torch.from_numpy(np.ascontiguousarray(t.esc).reshape(-1, ESCAPE_BUDGET))
        tensors[f"{name}.se12.fallback_bitmap"] = torch.from_numpy(np.ascontiguousarray(t.fallback_bitmap).reshape(-1))
        tensors[f"{name}.se12.fallback_raw"] = torch.from_numpy(np.ascontiguousarray(t.fallback_raw).reshape(-1))
        metadata[name] = _se12_metadata(t)
    payload = {"format": FORMAT_NAME, "format_version": CURRENT_FORMAT_VERSION, "tensors": metadata}
    path = pathlib.Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    st.torch.save_file(tensors, str(path), metadata={METADATA_KEY: json.dumps(payload)})


@dataclasses.dataclass(frozen=True)
class PackSummary:
    """Counts and eligible-tensor byte totals of a pack (pack_model.py:22-35)."""

    encoded: int
    passed_through: int
    original_bytes: int
    packed_bytes: int

    @property
    def ratio(self) -> float:
        return self.packed_bytes / self.original_bytes if self.original_bytes else 0.0


def _eligible(t: torch.Tensor) -> bool:
    return t.dtype == torch.bfloat16 and t.dim() == 2


def pack_model(model_dir: str | pathlib.Path, out_dir: str | pathlib.Path, device="cuda") -> PackSummary:
    """Packs every ``*.safetensors`` shard of ``model_dir`` into ``out_dir``
    (src/lws/application/codec/pack_model.py:65-80). SE12 encoding runs on
    the GPU; the written files are byte-identical to the reference packer's.
    The source files are only read."""
    from .codec import encode_device

    st = _safetensors()
    model_dir, out_dir = pathlib.Path(model_dir), pathlib.Path(out_dir)
    encoded = passed = original = packed = 0
    for shard_path in sorted(model_dir.glob(SHARD_GLOB)):
        entries = []
        with st.safe_open(str(shard_path), framework="pt") as shard:
            for name in shard.keys():
                t = shard.get_tensor(name)
                if _eligible(t):
                    host = encode_device(t.to(device)).to_tensor()
                    entries.append((name, host))
                    encoded += 1
                    original += t.numel() * 2
                    packed += byte_size(host)
                else:
                    entries.append((name, t))
                    passed += 1
        write_packed_shard(out_dir / shard_path.name, entries)
    return PackSummary(encoded, passed, original, packed)


# ---------------------------------------------------------------------- reading


def _packed_files(path: pathlib.Path) -> list:
    return sorted(path.glob(SHARD_GLOB)) if path.is_dir() else [path]


def _header(shard) -> dict:
    meta = shard.metadata() or {}
    if METADATA_KEY not in meta:
        raise ValueError("not an SE12 packed file: no 'se12' metadata")
    payload = json.loads(meta[METADATA_KEY])
    if payload.get("format") != FORMAT_NAME:
        raise ValueError(f"not an SE12 packed file: format {payload.get('format')!r}")
    validate_format_version(FormatVersion(int(payload.get("format_version", -1))))
    return payload["tensors"]


def read_packed(path: str | pathlib.Path) -> dict:
    """Reads a packed file or directory into host objects: name -> this
    package's ``Se12Tensor`` for SE12 entries, name -> torch tensor for
    pass-through entries. Raises ``UnsupportedFormatVersionError`` for an
    unknown format version (src/lws/domain/se12/container.py:21-27)."""
    st = _safetensors()
    out: dict = {}
    for f in _packed_files(pathlib.Path(path)):
        with st.safe_open(str(f), framework="pt") as shard:
            for name, meta in _header(shard).items():
                if not meta.get("eligible", False):
                    out[name] = shard.get_tensor(name)
                    continue
                if (meta["tile_rows"], meta["tile_cols"], meta["escape_budget"]) != (TILE_ROWS, TILE_COLS, ESCAPE_BUDGET):
                    raise ValueError(f"{name}: unsupported tiling {meta['tile_rows']}x{meta['tile_cols']}/{meta['escape_budget']}")
                streams = {s: shard.get_tensor(f"{name}.se12.{s}").numpy() for s in STREAM_SUFFIXES}
                rows, cols = meta["shape"]
                out[name] = make_tensor(rows, cols, meta["codebook"], streams["sm"], streams["ec"], streams["esc"],
                                        streams["fallback_bitmap"], streams["fallback_raw"])
    return out


def load_packed_tensors(path: str | pathlib.Path, device="cuda") -> dict:
    """``read_packed`` with every SE12 tensor uploaded as a ``DeviceSe12Matrix``
    and every pass-through tensor moved to ``device``."""
    from .device import DeviceSe12Matrix

    out = {}
    for name, value in read_packed(path).items():
        out[name] = DeviceSe12Matrix.from_tensor(value, device) if isinstance(value, Se12Tensor) else value.to(device)
    return out


__all__ = [
    "PackSummary",
    "UnsupportedFormatVersionError",
    "load_packed_tensors",
    "pack_model",
    "read_packed",
    "write_packed_shard",
]
