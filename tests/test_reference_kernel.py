"""The reference's own fused kernel, lws_gemv_se12 (compiled unchanged for
sm_100a into oracle/_ref by oracle/build_ref.py), run on this GPU: on the
GEMV parity shapes it can take (cols % 256 == 0, gemv_se12.cu:17-21) its output
is within 1e-3 of the fp64 oracle, like this package's kernel. Its launch
and side tables are the reference's (oracle/ref_gpu.py). This is the
comparison kernel bench.py's reference arm times; skipped when the library
was not built (no reference tree where build() ran)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
import ref_gpu
import se12_oracle as oracle

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-3
# (kind, rows, cols): the fused-GEMV parity shapes whose cols % 256 == 0
SHAPES = [("synthetic", 2304, 9216), ("synthetic", 2048, 2304), ("synthetic", 272, 2304), ("synthetic", 16, 65536),
          ("outliers", 64, 1024), ("outliers", 160, 2560), ("concentrated", 160, 2560), ("forced_fallback", 16, 256)]


def make_weights(kind, rows, cols):
    if kind == "synthetic":
        return cases.synthetic_weights(rows, cols, seed=rows * 7 + cols)
    if kind == "outliers":  # 1 % outliers x1024: most tiles fall back
        return cases.synthetic_weights(rows, cols, seed=4, outlier_rate=1e-2, outlier_scale=1024.0)
    if kind == "concentrated":
        return cases.concentrated(rows, cols, seed=5)
    return cases.forced_fallback_tile()


@pytest.fixture(scope="module", autouse=True)
def library():
    if not ref_gpu.available():
        pytest.skip("oracle/_ref/libref_kernels.so was not built")
    from se12_b200 import _build

    _build.build()
    torch.cuda.set_device(0)
    yield


@pytest.mark.parametrize("batch", [1, 3])
@pytest.mark.parametrize("kind,rows,cols", SHAPES)
def test_reference_kernel_matches_fp64_oracle(kind, rows, cols, batch):
    from se12_b200.device import DeviceSe12Matrix, stream_handle

    bits, rows, cols = make_weights(kind, rows, cols)
    bits = np.asarray(bits, dtype=np.uint16)
    s = oracle.encode(bits, rows, cols)

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(dtype)).cuda()

    m = DeviceSe12Matrix(s.rows, s.cols, s.codebook, up(s.sm, np.uint8), up(s.ec, np.uint8), up(s.esc, np.uint8),
                         up(s.fallback_bitmap, np.uint8), up(s.fallback_raw, np.int16))
    xb = oracle.bf16_round(np.random.default_rng(batch + rows).normal(size=(batch, cols)).astype(np.float32))
    x32 = torch.from_numpy(oracle.bits_to_float32(xb)).cuda().contiguous()
    y = torch.full((batch, rows), float("nan"), device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    ref_gpu.RefSe12Gemv(m, sms).launch(x32, y, stream_handle(torch.device("cuda", 0)))
    torch.cuda.synchronize()
    y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
    assert oracle.max_relative_error(y.cpu().numpy(), y64) <= TOLERANCE
    ours = m.gemv(torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()).cpu().numpy()
    assert oracle.max_relative_error(ours, y64) <= TOLERANCE
