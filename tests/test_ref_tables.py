"""The side tables the reference's GPU kernel reads, restated twice -- numpy
in the oracle (se12_oracle.row_escape_offset / fallback_offsets) and torch
in oracle/ref_gpu.py (what the GPU tests and the reference arm hand the
kernel) -- held to the reference's own host helpers
(src/lws/adapters/cuda/gemv.py:47-77) through
tests/golden/golden_ref_tables.json (make_ref_tables_golden.py), and the
reference's launch heuristic (src/lws/domain/launch/heuristic.py:46-51)."""

from __future__ import annotations

import hashlib
import json
import pathlib

import numpy as np
import pytest
import torch

import cases
import ref_gpu
import se12_oracle as oracle

GOLDEN = json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "golden_ref_tables.json").read_text())
CASES = cases.all_cases()


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", sorted(GOLDEN))
def test_side_tables_match_the_reference(name):
    bits, rows, cols = CASES[name]
    s = oracle.encode(np.asarray(bits, dtype=np.uint16), rows, cols)
    want = GOLDEN[name]
    reo = oracle.row_escape_offset(s)
    assert list(reo.shape) == want["row_escape_offset_shape"]
    assert digest(reo) == want["row_escape_offset"]
    assert digest(oracle.fallback_offsets(s)) == want["fallback_offsets"]
    tr, tc = reo.shape[0] // 16, reo.shape[1]
    ec = torch.from_numpy(np.ascontiguousarray(s.ec).reshape(-1))
    assert digest(ref_gpu.row_escape_offset(ec, tr, tc).numpy()) == want["row_escape_offset"]
    bm = torch.from_numpy(np.ascontiguousarray(s.fallback_bitmap).reshape(-1))
    assert digest(ref_gpu.fallback_offsets(bm, tr * tc).numpy()) == want["fallback_offsets"]


def test_default_launch_is_the_reference_heuristic():
    # (rows, batch) -> (blocks, threads) as the reference's
    # default_launch_configuration gives them for 148 SMs
    expected = {(256000, 1): (32000, 256), (2304, 1): (1152, 64), (1024, 1): (1024, 32), (100, 1): (100, 32),
                (4096, 16): (8192, 256)}
    for (rows, batch), want in expected.items():
        assert ref_gpu.default_launch(148, rows, batch) == want
