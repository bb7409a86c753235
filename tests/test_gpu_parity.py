"""Parity of the CUDA path (libse12_b200 through its C ABI) with the oracle.

* encoder: every stream byte-identical to the reference's (golden sha256);
* decode / decode_rows: bit-exact against the original weights;
* derived tables: escape positions and fallback ranks equal the oracle's;
* fused GEMV: max_i |y - y64| / max(|y64|, 1) <= 1e-3 against the fp64
  oracle (reference metric src/lws/bench/micro.py:154-159)
  for batch 1..20, padded and unpadded shapes, escape- and fallback-heavy
  matrices, and stream-K splits of every kind; deterministic across runs.
"""

from __future__ import annotations

import ctypes
import hashlib

import numpy as np
import pytest
import torch

import cases
import se12_oracle as oracle

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-3
STREAMS = ("sm", "ec", "esc", "fallback_bitmap", "fallback_raw")


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module", autouse=True)
def library():
    from se12_b200 import _build

    _build.build()
    torch.cuda.set_device(0)
    yield
    from se12_b200.device import device_status

    assert device_status() == 0, "a kernel raised the device status word"


def device_matrix(streams: oracle.Streams):
    from se12_b200.device import DeviceSe12Matrix

    dev = torch.device("cuda", 0)

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(dtype)).to(dev)

    return DeviceSe12Matrix(streams.rows, streams.cols, streams.codebook, up(streams.sm, np.uint8), up(streams.ec, np.uint8),
                            up(streams.esc, np.uint8), up(streams.fallback_bitmap, np.uint8), up(streams.fallback_raw, np.int16))


def reference_streams(name, golden_table, golden_arrays, golden_cases) -> oracle.Streams:
    """The reference's own streams when committed, else the (pinned) oracle's."""
    bits, rows, cols = golden_cases[name]
    entry = golden_table[name]
    if entry["stored_in_npz"]:
        return oracle.Streams(rows=rows, cols=cols, codebook=tuple(entry["codebook"]),
                              **{k: golden_arrays[f"{name}/{k}"] for k in STREAMS})
    streams = oracle.encode(bits, rows, cols)
    assert sha(streams.sm) == entry["streams"]["sm"]["sha256"]
    return streams


ALL_CASES = sorted(cases.all_cases())


@pytest.mark.parametrize("name", ALL_CASES)
def test_gpu_encoder_is_byte_identical_to_reference(name, golden_table, golden_cases):
    from se12_b200.codec import encode_device

    bits, rows, cols = golden_cases[name]
    w = torch.from_numpy(np.asarray(bits, dtype=np.uint16).view(np.int16).reshape(rows, cols).copy()).view(torch.bfloat16).cuda()
    m = encode_device(w)
    t = m.to_tensor()
    entry = golden_table[name]
    assert list(t.codebook) == entry["codebook"]
    got = {"sm": t.sm, "ec": t.ec, "esc": t.esc, "fallback_bitmap": t.fallback_bitmap, "fallback_raw": t.fallback_raw}
    for key in STREAMS:
        assert list(got[key].shape) == entry["streams"][key]["shape"], key
        assert sha(got[key]) == entry["streams"][key]["sha256"], f"{name}: {key} differs from the reference encoder"
    assert m.byte_size == entry["byte_size"]


@pytest.mark.parametrize("name", ALL_CASES)
def test_gpu_decode_is_bit_exact(name, golden_table, golden_arrays, golden_cases):
    bits, rows, cols = golden_cases[name]
    streams = reference_streams(name, golden_table, golden_arrays, golden_cases)
    m = device_matrix(streams)
    out = m.decode().view(torch.int16).cpu().numpy().reshape(-1).view(np.uint16)
    assert np.array_equal(out, np.asarray(bits, dtype=np.uint16))
    # derived tables
    assert np.array_equal(m.escape_pos.cpu().numpy().view(np.uint16).reshape(-1, 16), oracle.escape_positions(streams))
    fb = oracle.fallback_mask(streams)
    expect = np.where(fb, oracle.fallback_offsets(streams), -1)
    index = m.fallback_index.cpu().numpy()
    assert index.size == (expect.size + 3) // 4 * 4
    assert np.array_equal(index[:expect.size], expect) and np.all(index[expect.size:] == -1)


def test_gpu_decode_rows_in_request_order(golden_cases):
    bits, rows, cols = cases.synthetic_weights(48, 512, seed=4, outlier_rate=5e-3, outlier_scale=512.0)
    streams = oracle.encode(bits, rows, cols)
    m = device_matrix(streams)
    request = [5, 0, 47, 12, 12, 33]
    got = m.decode_rows(request).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, oracle.decode_rows(streams, request))


def test_decoder_adapter_interface(golden_cases):
    from se12_b200.decoder import CudaSe12WeightDecoder, RowIndices
    from se12_b200.format import as_tensor, make_tensor

    bits, rows, cols = golden_cases["gpu_decode_random_64x512"]
    s = oracle.encode(bits, rows, cols)
    t = make_tensor(s.rows, s.cols, s.codebook, s.sm, s.ec, s.esc, s.fallback_bitmap, s.fallback_raw)
    dec = CudaSe12WeightDecoder(None, None)
    assert np.array_equal(dec.decode(t).bit_pattern.view(np.uint16), np.asarray(bits, dtype=np.uint16))
    part = dec.decode_rows(as_tensor(t), RowIndices(values=(5, 0, 63)))
    assert np.array_equal(part.bit_pattern.view(np.uint16), np.asarray(bits, dtype=np.uint16).reshape(rows, cols)[[5, 0, 63]].reshape(-1))
    assert dec.decode_to_device(t).dtype == torch.bfloat16


# ------------------------------------------------------------------ GEMV

GEMV_SHAPES = [
    ("synthetic", 2304, 9216),     # config 0: rows split between CTAs (stream-K fixup)
    ("synthetic", 2048, 2304),     # Gemma-2-2B q_proj
    ("synthetic", 272, 2304),
    ("synthetic", 32, 2560),       # fewer tiles than CTAs: every row shared by 10 CTAs
    ("synthetic", 16, 65536),      # one row of 256 tiles over 64 CTAs: 63 contributors per split row
    ("synthetic", 33, 300),        # padding in both directions, K % 8 != 0
    ("synthetic", 1, 1),
    ("synthetic", 36, 1),
    ("synthetic", 100, 264),
    ("outliers", 64, 1024),        # 1% outliers x1024: 13 of 16 tiles fall back
    ("outliers", 160, 2560),
    ("concentrated", 160, 2560),
    ("forced_fallback", 16, 256),
    # shapes that reach the remaining launch configurations (checked by
    # test_launch_table_reaches_every_configuration on a 148-SM B200)
    ("synthetic", 16, 4608),       # 4-tile stages, stream-K, x resident (batch 1) / staged (batch 4)
    ("synthetic", 16, 3584),       # 4-tile stages, row mode, staged x (batch 8)
    ("synthetic", 1024, 5120),     # 8-tile stages, stream-K (batch 1)
    ("synthetic", 4096, 1792),     # 8-tile stages, one CTA per SM (batch 16)
    # staged x with a ragged last tile column (batch >= 4 / 8): whole tiles by
    # bulk copy, the last one by cp.async with zeros past K (K % 8 != 0 too)
    ("synthetic", 16, 20000),
    ("synthetic", 32, 12300),
    ("synthetic", 4816, 2304),     # the wide layout (batch 4, 8)
]


def make_weights(kind, rows, cols):
    if kind == "synthetic":
        return cases.synthetic_weights(rows, cols, seed=rows * 7 + cols)
    if kind == "outliers":
        return cases.synthetic_weights(rows, cols, seed=4, outlier_rate=1e-2, outlier_scale=1024.0)
    if kind == "concentrated":
        return cases.concentrated(rows, cols, seed=5)
    return cases.forced_fallback_tile()


def activations(batch, cols, seed=1):
    x = np.random.default_rng(seed).normal(0.0, 1.0, size=(batch, cols)).astype(np.float32)
    return oracle.bf16_round(x)


_matrices: dict = {}


def gemv_fixture(kind, rows, cols):
    key = (kind, rows, cols)
    if key not in _matrices:
        bits, r, c = make_weights(kind, rows, cols)
        streams = oracle.encode(bits, r, c)
        _matrices[key] = (bits, streams, device_matrix(streams))
    return _matrices[key]


@pytest.mark.parametrize("kind,rows,cols", GEMV_SHAPES)
@pytest.mark.parametrize("batch", [1, 2, 4, 8, 16])
def test_fused_gemv_matches_fp64_oracle(kind, rows, cols, batch):
    bits, streams, m = gemv_fixture(kind, rows, cols)
    xb = activations(batch, cols)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = m.gemv(x).cpu().numpy()
    y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
    err = oracle.max_relative_error(y, y64)
    assert y.shape == (batch, rows)
    assert err <= TOLERANCE, f"max rel err {err:.3e}"
    # the reference CPU path (numpy decode + fp32 matmul) is held to the same bar
    y_cpu = oracle.gemv_reference_cpu(streams, oracle.bits_to_float32(xb))
    assert oracle.max_relative_error(y_cpu, y64) <= TOLERANCE


def test_launch_table_reaches_every_configuration():
    """The parity shapes above run every kernel configuration: 4-tile stages
    with x resident or staged, 8-tile stages (x always resident), each in row
    mode and stream-K, pipelines deeper than 2 stages, and the
    wide layout (one CTA per SM, x resident, 4-tile stages taken in turn by
    its warp groups; row mode only). Configurations with one CTA per SM run
    the kernel builds made for one CTA per SM (more registers): the shapes
    reach each of them (8-tile stages at batch <= 8; 4-tile stages with x
    resident or staged and 8-tile stages at batch 9..16)."""
    from se12_b200 import _lib

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    seen, deep, solo = set(), False, set()
    for kind, rows, cols in GEMV_SHAPES:
        m = gemv_fixture(kind, rows, cols)[2]
        for batch in (1, 2, 4, 8, 16):
            c = m.launch_config(batch)
            # the host-only plan from the shape gives the same answer
            cfg = _lib.Se12LaunchConfigStruct()
            assert _lib.load().se12_gemv_plan(rows, cols, batch, sms, ctypes.byref(cfg)) == 0
            assert {name: getattr(cfg, name) for name, _ in cfg._fields_} == c
            if c["wide"]:
                assert c["threads"] == 576 and c["stage_tiles"] == 4 and c["x_resident"] == 1 and c["stages"] >= 6
                assert c["ctas_per_sm"] == 1 and 1 <= c["grid"] <= sms and batch <= 8 and c["row_mode"] == 1
            else:
                assert c["threads"] == 320 and 1 <= c["grid"] <= 2 * sms
            layout = "wide" if c["wide"] else c["stage_tiles"]
            seen.add((layout, c["x_resident"], c["row_mode"]))
            if not c["wide"] and c["ctas_per_sm"] == 1:
                solo.add((1 if batch <= 8 else 2, c["stage_tiles"], c["x_resident"]))
            deep = deep or c["stages"] > 2
    if sms != 148:
        pytest.skip("the shapes are chosen for 148 SMs")
    assert all(x == 1 for t, x, _ in seen if t in (8, "wide")), "8-tile stages or the wide layout with staged x"
    missing = {(4, x, r) for x in (0, 1) for r in (0, 1)} | {(8, 1, r) for r in (0, 1)} | {("wide", 1, 1)}
    missing -= seen
    assert not missing, f"configurations no parity shape reaches: {sorted(missing, key=str)}"
    assert deep
    assert solo >= {(1, 8, 1), (2, 4, 0), (2, 4, 1), (2, 8, 1)}, sorted(solo)


@pytest.mark.parametrize("batch", [3, 9, 20])
def test_fused_gemv_odd_and_chunked_batches(batch):
    bits, streams, m = gemv_fixture("synthetic", 272, 2304)
    xb = activations(batch, 2304, seed=batch)
    y = m.gemv(torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()).cpu().numpy()
    y64 = oracle.gemv_fp64(bits, 272, 2304, oracle.bits_to_float32(xb))
    assert oracle.max_relative_error(y, y64) <= TOLERANCE


def test_fused_gemv_fp32_activations():
    bits, streams, m = gemv_fixture("synthetic", 2048, 2304)
    x = np.random.default_rng(3).normal(0.0, 1.0, size=(4, 2304)).astype(np.float32)
    y = m.gemv(torch.from_numpy(x).cuda()).cpu().numpy()
    y64 = oracle.gemv_fp64(bits, 2048, 2304, x)
    assert oracle.max_relative_error(y, y64) <= 1e-5


def test_fused_gemv_is_deterministic():
    bits, streams, m = gemv_fixture("synthetic", 2304, 9216)
    x = torch.from_numpy(activations(4, 9216).view(np.int16)).view(torch.bfloat16).cuda()
    first = m.gemv(x).clone()
    for _ in range(3):
        assert torch.equal(m.gemv(x), first)


@pytest.mark.parametrize("cols", [300, 1000, 2311])
def test_fused_gemv_ignores_x_past_cols(cols):
    """x[b, cols..ldx) may hold anything (NaN here): the result must not see it."""
    bits, rows, _ = cases.synthetic_weights(48, cols, seed=cols)
    m = device_matrix(oracle.encode(bits, rows, cols))
    xb = activations(3, cols, seed=cols)
    ldx = (cols + 7) // 8 * 8 + 16
    x = torch.full((3, ldx), float("nan"), dtype=torch.bfloat16, device="cuda")
    x[:, :cols] = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = m.gemv(x[:, :cols]).cpu().numpy()
    y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
    assert np.isfinite(y).all()
    assert oracle.max_relative_error(y, y64) <= TOLERANCE


def test_fused_gemv_with_infinite_padding_weight():
    """codebook[0] == 255: the padding weights (+0.0, code 0) would decode to
    +inf; rows of finite weights must still match the oracle."""
    rows, cols = 64, 300
    w = np.random.default_rng(9).normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
    w[:40, :] = np.inf  # 12000 of 19200 weights: the most frequent exponent is 255
    bits = oracle.bf16_round(w).reshape(-1)
    streams = oracle.encode(bits, rows, cols)
    assert streams.codebook[0] == 255
    m = device_matrix(streams)
    xb = oracle.bf16_round(np.abs(np.random.default_rng(2).normal(0.0, 1.0, size=(2, cols))) + 0.01)
    y = m.gemv(torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()).cpu().numpy()
    y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
    assert np.isposinf(y[:, :40]).all()
    assert oracle.max_relative_error(y[:, 40:], y64[:, 40:]) <= TOLERANCE


def test_matvec_adapter_interface():
    from se12_b200.format import make_tensor
    from se12_b200.gemv import RawBf16MatVecKernel, Se12MatVecKernel

    bits, rows, cols = cases.synthetic_weights(512, 2304, seed=9)
    s = oracle.encode(bits, rows, cols)
    tensor = make_tensor(s.rows, s.cols, s.codebook, s.sm, s.ec, s.esc, s.fallback_bitmap, s.fallback_raw)
    fused = Se12MatVecKernel(None, None, tensor, 148)
    w = torch.from_numpy(np.asarray(bits, dtype=np.uint16).view(np.int16).reshape(rows, cols)).view(torch.bfloat16)
    raw = RawBf16MatVecKernel(None, None, w, 148)
    x = torch.randn(4, cols, dtype=torch.bfloat16, device="cuda")
    y64 = oracle.gemv_fp64(bits, rows, cols, x.float().cpu().numpy())
    for kernel in (fused, raw):
        y = kernel.multiply(x)
        assert y.dtype == torch.float32 and tuple(y.shape) == (4, rows)
        assert oracle.max_relative_error(y.cpu().numpy(), y64) <= TOLERANCE


@pytest.mark.parametrize("rows,cols", [(2304, 9216), (33, 300), (256, 2304), (9216, 2304)])
@pytest.mark.parametrize("batch", [1, 8, 16])
def test_dense_bf16_baseline_matches_fp64(rows, cols, batch):
    from se12_b200.device import bf16_gemv

    bits, _, _ = cases.synthetic_weights(rows, cols, seed=11)
    w = torch.from_numpy(np.asarray(bits, dtype=np.uint16).view(np.int16).reshape(rows, cols)).view(torch.bfloat16).cuda()
    xb = activations(batch, cols, seed=2)
    y = bf16_gemv(w, torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()).cpu().numpy()
    y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
    assert oracle.max_relative_error(y, y64) <= TOLERANCE


def test_round_trip_through_codec_api():
    from se12_b200.codec import decode_tensor, encode_tensor
    from se12_b200.format import Bf16Weights, MatrixShape

    bits, rows, cols = cases.synthetic_weights(96, 768, seed=21)
    weights = Bf16Weights(bit_pattern=np.asarray(bits, dtype=np.uint16).view(np.int16))
    encoded = encode_tensor(weights, MatrixShape(rows, cols))
    ref = oracle.encode(bits, rows, cols)
    assert encoded.codebook == ref.codebook
    assert np.array_equal(encoded.sm, ref.sm) and np.array_equal(encoded.ec, ref.ec) and np.array_equal(encoded.esc, ref.esc)
    assert np.array_equal(decode_tensor(encoded).bit_pattern, weights.bit_pattern)


def test_shared_workspace_across_interleaved_matrices():
    """Calls on one stream share one workspace; interleaving matrices of
    different tile-row counts must not disturb the stream-K counters."""
    shapes = [("synthetic", 2304, 9216), ("concentrated", 160, 2560), ("synthetic", 33, 300), ("synthetic", 2048, 2304)]
    expected = {}
    for kind, rows, cols in shapes:
        bits, _, m = gemv_fixture(kind, rows, cols)
        xb = activations(2, cols, seed=rows)
        expected[(kind, rows, cols)] = (m, torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda(),
                                        oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb)))
    for _ in range(3):
        for key in shapes + shapes[::-1]:
            m, x, y64 = expected[key]
            assert oracle.max_relative_error(m.gemv(x).cpu().numpy(), y64) <= TOLERANCE, key
