"""The CPU oracle against fixtures produced by the reference codec itself.

Every stream, the codebook, the packed byte count, the fallback offsets and
the decoded bits of every golden case must match the reference byte for byte
(tests/golden/make_golden.py ran src/lws/domain/se12/codec.py to make them).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

import se12_oracle as oracle

STREAM_NAMES = ("sm", "ec", "esc", "fallback_bitmap", "fallback_raw")


def _sha(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def _streams_as_arrays(streams):
    return {
        "sm": streams.sm,
        "ec": streams.ec,
        "esc": streams.esc,
        "fallback_bitmap": streams.fallback_bitmap,
        "fallback_raw": streams.fallback_raw,
    }


def test_every_golden_case_is_present(golden_table, golden_cases):
    assert set(golden_table) == set(golden_cases)


@pytest.mark.parametrize("name", sorted(__import__("cases").all_cases()))
def test_oracle_encode_decode_matches_reference(name, golden_table, golden_arrays, golden_cases):
    bits, rows, cols = golden_cases[name]
    entry = golden_table[name]
    assert _sha(np.asarray(bits, dtype=np.uint16).view(np.int16)) == entry["input_sha256"], "input recipe drifted"

    streams = oracle.encode(bits, rows, cols)
    assert list(streams.codebook) == entry["codebook"]
    arrays = _streams_as_arrays(streams)
    for key in STREAM_NAMES:
        meta = entry["streams"][key]
        assert str(arrays[key].dtype) == meta["dtype"], key
        assert list(arrays[key].shape) == meta["shape"], key
        assert _sha(arrays[key]) == meta["sha256"], f"{name}: stream {key} differs from the reference"
        if entry["stored_in_npz"]:
            assert np.array_equal(arrays[key], golden_arrays[f"{name}/{key}"])
    assert oracle.byte_size(streams) == entry["byte_size"]
    assert int(oracle.fallback_mask(streams).sum()) == entry["fallback_tiles"]
    assert _sha(oracle.fallback_offsets(streams)) == entry["fallback_offsets_sha256"]

    decoded = oracle.decode(streams)
    assert _sha(decoded.reshape(-1).view(np.int16)) == entry["decoded_sha256"]
    assert np.array_equal(decoded.reshape(-1), np.asarray(bits, dtype=np.uint16))


def test_oracle_decodes_the_reference_streams(golden_table, golden_arrays, golden_cases):
    """Decode streams written by the reference (not by the oracle's encoder)."""
    for name, entry in golden_table.items():
        if not entry["stored_in_npz"]:
            continue
        bits, rows, cols = golden_cases[name]
        streams = oracle.Streams(
            rows=rows,
            cols=cols,
            codebook=tuple(entry["codebook"]),
            **{key: golden_arrays[f"{name}/{key}"] for key in STREAM_NAMES},
        )
        assert np.array_equal(oracle.decode(streams).reshape(-1), np.asarray(bits, dtype=np.uint16)), name


def test_escape_positions_recover_every_escape():
    bits, rows, cols = __import__("cases").synthetic_weights(64, 1024, seed=4, outlier_rate=1e-2, outlier_scale=1024.0)
    streams = oracle.encode(bits, rows, cols)
    pos = oracle.escape_positions(streams)
    fb = oracle.fallback_mask(streams)
    exp, _ = oracle.split_bits(oracle.decode(streams))
    padded = np.zeros(oracle.padded_shape(rows, cols), dtype=np.uint8)
    padded[:rows, :cols] = exp
    tiles = oracle.to_tiles(padded).reshape(streams.tile_count, -1)
    for tile in range(streams.tile_count):
        used = pos[tile][pos[tile] != 0xFFFF]
        if fb[tile]:
            assert used.size == 0
            continue
        assert np.all(np.diff(used.astype(np.int64)) > 0)
        assert np.array_equal(tiles[tile][used], streams.esc[tile][: used.size])


def test_bf16_round_matches_torch():
    import torch

    values = np.random.default_rng(0).normal(0, 3, size=4096).astype(np.float32)
    values[:4] = [np.inf, -np.inf, 0.0, -0.0]
    ours = oracle.bf16_round(values)
    theirs = torch.from_numpy(values).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


def test_error_metric_matches_reference_definition():
    y64 = np.array([0.5, -3.0, 100.0])
    y = y64 + np.array([1e-4, 3e-3, 0.2])
    assert oracle.max_relative_error(y, y64) == pytest.approx(max(1e-4 / 1.0, 3e-3 / 3.0, 0.2 / 100.0))
