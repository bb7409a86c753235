"""Segmented matrices: several SE12 matrices with the same columns (q/k/v,
gate/up) concatenated tile-major so that one fused GEMV computes them all,
each segment decoding with its own codebook.

Parity: the GEMV of the segmented matrix equals, segment by segment, the
fp64 oracle of each matrix within max_i |y - y64| / max(|y64|, 1) <= 1e-3;
its decode is bit-exact against each matrix's oracle decode.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
import se12_oracle as oracle

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-3


@pytest.fixture(scope="module", autouse=True)
def library():
    from se12_b200 import _build

    _build.build()
    torch.cuda.set_device(0)
    yield


def device_matrix(streams: oracle.Streams):
    from se12_b200.device import DeviceSe12Matrix

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(dtype)).cuda()

    return DeviceSe12Matrix(streams.rows, streams.cols, streams.codebook, up(streams.sm, np.uint8), up(streams.ec, np.uint8),
                            up(streams.esc, np.uint8), up(streams.fallback_bitmap, np.uint8), up(streams.fallback_raw, np.int16))


def infinite_padding_bits(rows: int, cols: int):
    """Most frequent exponent 255 (codebook[0] == 255): padding weights would decode to +inf."""
    w = np.random.default_rng(9).normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
    w[: rows * 5 // 8, :] = np.inf
    return oracle.bf16_round(w).reshape(-1)


def segment_bits(kind: str, rows: int, cols: int):
    if kind == "plain":
        return cases.synthetic_weights(rows, cols, seed=rows + cols)[0]
    if kind == "wide":  # another exponent range, so another codebook
        return cases.synthetic_weights(rows, cols, seed=3 * rows + cols, sigma=4.0)[0]
    if kind == "outliers":  # 1 % outliers x1024: most tiles fall back
        return cases.synthetic_weights(rows, cols, seed=4, outlier_rate=1e-2, outlier_scale=1024.0)[0]
    return infinite_padding_bits(rows, cols)


SEGMENT_SETS = [
    [("plain", 64), ("outliers", 32), ("wide", 33)],                     # ragged last segment
    [("wide", 16), ("infinite", 64), ("outliers", 48), ("plain", 100)],  # four segments
    [("plain", 2048), ("wide", 1024), ("plain", 1024)],                  # q/k/v of Gemma-2-2B
]


def build(spec, cols):
    from se12_b200.device import DeviceSe12Matrix

    parts = []
    for kind, rows in spec:
        bits = segment_bits(kind, rows, cols)
        streams = oracle.encode(bits, rows, cols)
        parts.append((bits, rows, streams, device_matrix(streams)))
    return parts, DeviceSe12Matrix.concatenate([p[3] for p in parts])


@pytest.mark.parametrize("spec", range(len(SEGMENT_SETS)))
@pytest.mark.parametrize("cols", [300, 2304])
@pytest.mark.parametrize("batch", [1, 5, 16])
def test_segmented_gemv_matches_each_segment(spec, cols, batch):
    parts, seg = build(SEGMENT_SETS[spec], cols)
    assert len({p[2].codebook for p in parts}) > 1, "the segments should not share one codebook"
    xb = oracle.bf16_round(np.abs(np.random.default_rng(batch).normal(0.0, 1.0, size=(batch, cols))) + 0.01)
    y = seg.gemv(torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()).cpu().numpy()
    assert y.shape == (batch, sum(p[1] for p in parts))
    r0 = 0
    for bits, rows, streams, _ in parts:
        y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
        ys = y[:, r0:r0 + rows]
        finite = np.isfinite(y64).all(axis=0)
        assert np.array_equal(np.isposinf(ys[:, ~finite]), np.isposinf(y64[:, ~finite]))
        assert oracle.max_relative_error(ys[:, finite], y64[:, finite]) <= TOLERANCE, (streams.codebook[0], rows)
        r0 += rows


@pytest.mark.parametrize("cols", [300, 2304])
def test_segmented_decode_is_bit_exact(cols):
    parts, seg = build(SEGMENT_SETS[1], cols)
    want = np.concatenate([oracle.decode(p[2]).reshape(p[1], cols) for p in parts]).view(np.uint16)
    got = seg.decode().view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, want)
    rows = [0, 17, 16 + 64 + 5, want.shape[0] - 1]
    part = seg.decode_rows(rows).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(part, want[rows])


def test_segmented_matrix_keeps_the_byte_count_of_its_parts():
    parts, seg = build(SEGMENT_SETS[0], 2304)
    assert seg.byte_size == sum(p[3].byte_size for p in parts)
    assert seg.tiles == sum(p[3].tiles for p in parts)
    assert seg.fallback_tiles == sum(p[3].fallback_tiles for p in parts) > 0
    for part, back in zip(parts, seg.segment_tensors()):  # the segments come back as the tensors given
        want = part[3].to_tensor()
        assert (back.rows, back.cols, back.codebook) == (want.rows, want.cols, want.codebook)
        for name in ("sm", "ec", "esc", "fallback_bitmap", "fallback_raw"):
            assert np.array_equal(np.asarray(getattr(back, name)).reshape(-1), np.asarray(getattr(want, name)).reshape(-1)), name


def test_concatenate_rejects_what_cannot_be_one_matrix():
    from se12_b200.device import DeviceSe12Matrix

    a = device_matrix(oracle.encode(segment_bits("plain", 40, 300), 40, 300))
    b = device_matrix(oracle.encode(segment_bits("plain", 32, 300), 32, 300))
    c = device_matrix(oracle.encode(segment_bits("plain", 32, 512), 32, 512))
    with pytest.raises(ValueError, match="multiple of 16"):
        DeviceSe12Matrix.concatenate([a, b])
    with pytest.raises(ValueError, match="same columns"):
        DeviceSe12Matrix.concatenate([b, c])
    with pytest.raises(ValueError, match="at most 4"):
        DeviceSe12Matrix.concatenate([b, b, b, b, b])
    assert DeviceSe12Matrix.concatenate([b, a]).rows == 72
