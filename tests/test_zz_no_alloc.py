"""se12_gemv_noalloc (the GEMV variant whose scratch is a fixed array in the
library's device image) against se12_gemv (caller workspace), through the
C ABI: two calls in a row per case, each within the GEMV tolerance
max_i |y - y_ref| / max(|y_ref|, 1) <= 1e-3 of the workspace entry point.

This file is collected last on purpose: it must pass both alone in a fresh
process (the first call on the device sets the scratch up) and after every
other GPU test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-3


@pytest.fixture(scope="module", autouse=True)
def library():
    from se12_b200 import _build

    _build.build()
    torch.cuda.set_device(0)
    yield


def synthetic_bf16(rows: int, cols: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
    outliers = torch.rand(rows, cols, generator=g, device="cuda") < 1e-4
    return torch.where(outliers, w * 64, w).to(torch.bfloat16)


def noalloc_gemv(m, x: torch.Tensor, y: torch.Tensor) -> int:
    from se12_b200 import _lib
    from se12_b200.device import stream_handle

    lib = _lib.load()
    return lib.se12_gemv_noalloc(m.handle, ctypes.c_void_p(x.data_ptr()), x.shape[0], x.stride(0),
                                 ctypes.c_void_p(y.data_ptr()), y.stride(0), ctypes.c_void_p(stream_handle(x.device)))


def rel_err(y: torch.Tensor, ref: torch.Tensor) -> float:
    return float(((y.double() - ref.double()).abs() / ref.double().abs().clamp_min(1.0)).max())


# (rows, cols, batch, stream-K?): the stream-K cases split tile rows between
# CTAs, so their partial rows and per-CTA flags go through the fixed scratch
# (written by the contributors, read and cleared by the finisher); the row
# mode cases never touch it.
CASES = [
    (2304, 2304, 1, False),
    (2304, 2304, 4, False),
    (1000, 700, 3, False),
    (4608, 9216, 16, False),
    (256, 9216, 1, True),     # 144 CTAs, x resident
    (1024, 16384, 4, True),   # 296 CTAs (two per SM), x staged
    (256, 9216, 16, True),    # two batch blocks through the partial rows
]


@pytest.mark.parametrize("rows,cols,batch,stream_k", CASES)
def test_noalloc_matches_workspace_entry_point_on_two_calls(rows, cols, batch, stream_k):
    from se12_b200 import _lib
    from se12_b200.codec import encode_device
    from se12_b200.device import device_status

    m = encode_device(synthetic_bf16(rows, cols, seed=rows + cols))
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert m.launch_config(batch)["row_mode"] == (0 if stream_k else 1)
    ldx = (cols + 7) // 8 * 8
    for call in range(2):
        g = torch.Generator(device="cuda").manual_seed(1000 * call + batch)
        xs = torch.zeros(batch, ldx, dtype=torch.bfloat16, device="cuda")
        xs[:, :cols] = torch.randn(batch, cols, generator=g, device="cuda").to(torch.bfloat16)
        y_ref = m.gemv(xs[:, :cols])
        y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
        _lib.check(noalloc_gemv(m, xs, y), "se12_gemv_noalloc")
        torch.cuda.synchronize()
        assert device_status() == 0
        err = rel_err(y, y_ref)
        assert err <= TOLERANCE, f"call {call}: max rel err {err:.3g} against se12_gemv"


def test_noalloc_rejects_a_batch_beyond_its_scratch():
    from se12_b200 import _lib
    from se12_b200.codec import encode_device

    m = encode_device(synthetic_bf16(64, 512, seed=3))
    x = torch.zeros(17, 512, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(17, 64, dtype=torch.float32, device="cuda")
    status = noalloc_gemv(m, x, y)
    assert status == 1  # SE12_ERR_INVALID_ARGUMENT, nothing launched
    assert "batch must be in 1..16" in _lib.load().se12_last_error().decode()


def test_noalloc_serves_more_than_a_million_rows():
    """The scratch does not depend on the matrix: 65537 tile rows work."""
    from se12_b200 import _lib
    from se12_b200.device import DeviceSe12Matrix

    rows, cols = 65537 * 16, 256
    tiles = 65537
    dev = torch.device("cuda", 0)
    zeros = lambda n, dtype=torch.uint8: torch.zeros(n, dtype=dtype, device=dev)  # noqa: E731
    # every weight decodes to +2^(100 - 127): code 0, sign/mantissa 0
    m = DeviceSe12Matrix(rows, cols, tuple(range(100, 115)), zeros(tiles * 4096), zeros(tiles * 2048), zeros(tiles * 16),
                         zeros((tiles + 7) // 8), zeros(0, torch.int16))
    x = torch.randn(2, cols, device=dev).to(torch.bfloat16)
    y_ref = m.gemv(x)
    for call in range(2):
        y = torch.full((2, rows), float("nan"), dtype=torch.float32, device=dev)
        _lib.check(noalloc_gemv(m, x, y), "se12_gemv_noalloc")
        torch.cuda.synchronize()
        assert rel_err(y, y_ref) <= TOLERANCE, f"call {call}"
