"""Seeded input recipes for the SE12 golden fixtures.

Each recipe rebuilds, draw for draw, an input that the reference's own tests
or benchmark use (file:line given per case), so the fixtures produced by
``make_golden.py`` (which runs the reference codec on these inputs) pin the
oracle and the CUDA kernels to the reference's behaviour.

Every function returns ``(bits_uint16[rows*cols], rows, cols)``.
"""

from __future__ import annotations

import numpy as np


def _bits(sign: int, exponent: int, mantissa: int) -> int:
    return (sign << 15) | (exponent << 7) | mantissa


def float_edge_cases():
    """+-0, subnormals, +-inf, NaN payloads, extreme normals, then 200 random
    normals (tests/test_spec_se12_roundtrip.py:36-64, seed 7)."""
    edge = [
        _bits(0, 0, 0), _bits(1, 0, 0), _bits(0, 0, 1), _bits(1, 0, 1), _bits(0, 0, 0x7F),
        _bits(0, 0xFF, 0), _bits(1, 0xFF, 0), _bits(0, 0xFF, 0x40), _bits(0, 0xFF, 0x7F), _bits(1, 0xFF, 0x01),
        _bits(0, 1, 0), _bits(1, 1, 0), _bits(0, 0xFE, 0x7F), _bits(1, 0xFE, 0x7F),
    ]
    rng = np.random.default_rng(7)
    normals = [_bits(int(rng.integers(0, 2)), int(rng.integers(1, 0xFE)), int(rng.integers(0, 0x80))) for _ in range(200)]
    values = np.array(edge + normals, dtype=np.uint16)
    return values, 1, values.size


RANDOM_SHAPES = ((16, 256), (32, 256), (16, 512), (32, 512), (33, 300), (1, 1), (36, 1), (160, 2560))


def random_bit_shapes():
    """Uniform random 16-bit patterns over padded and unpadded shapes, one
    generator for all shapes in order (tests/test_spec_se12_roundtrip.py:67-75,
    seed 11). Yields one case per shape."""
    rng = np.random.default_rng(11)
    for rows, cols in RANDOM_SHAPES:
        bits = rng.integers(0, 65536, size=rows * cols, dtype=np.uint32).astype(np.uint16)
        yield bits, rows, cols


def forced_fallback_tile():
    """One 16x256 tile with 20 distinct rare exponents beyond 15 dominant ones
    (tests/test_spec_se12_roundtrip.py:78-102, seed 3)."""
    rng = np.random.default_rng(3)
    n = 16 * 256
    overflow = 20
    exponents = np.zeros(n, dtype=np.uint8)
    fill = n - overflow
    exponents[:fill] = np.tile(np.arange(15, dtype=np.uint8), fill // 15 + 1)[:fill]
    exponents[fill:] = np.arange(100, 100 + overflow, dtype=np.uint8)
    sign = rng.integers(0, 2, size=n).astype(np.uint16)
    mantissa = rng.integers(0, 0x80, size=n).astype(np.uint16)
    return (sign << 15) | (exponents.astype(np.uint16) << 7) | mantissa, 16, 256


def concentrated(rows: int, cols: int, seed: int, low: int = 120, high: int = 135):
    """Exponents drawn uniformly from [low, high): every tile fits its escape
    budget (tests/test_spec_se12_roundtrip.py:105-119 with 160x2560 seed 5;
    tests/test_spec_fused_gemv.py:28-35 with 32x512 seed 1;
    tests/test_spec_pack.py:33-46 with 64x512 seed 1 and 32x256 seed 2)."""
    rng = np.random.default_rng(seed)
    n = rows * cols
    exponents = rng.choice(np.arange(low, high, dtype=np.uint8), size=n)
    sign = rng.integers(0, 2, size=n).astype(np.uint16)
    mantissa = rng.integers(0, 0x80, size=n).astype(np.uint16)
    return (sign << 15) | (exponents.astype(np.uint16) << 7) | mantissa, rows, cols


def gpu_decode_random():
    """64x512 uniform random bits (tests/test_spec_gpu_decode.py:33-36,100-103, seed 7)."""
    rng = np.random.default_rng(7)
    bits = rng.integers(0, 65536, size=64 * 512, dtype=np.uint32).astype(np.uint16)
    return bits, 64, 512


def synthetic_weights(rows: int, cols: int, seed: int = 0, sigma: float = 0.02, outlier_rate: float = 1e-4, outlier_scale: float = 64.0, zero_rate: float = 1e-3):
    """The benchmark distribution: N(0, sigma) cast to BF16 (round to nearest
    even), then ``outlier_rate`` of the entries scaled by ``outlier_scale``,
    then ``zero_rate`` of them set to exact +-0 (sign 50/50)."""
    rng = np.random.default_rng(seed)
    values = rng.normal(0.0, sigma, size=(rows, cols)).astype(np.float32).reshape(-1)
    n = values.size
    n_out = int(round(outlier_rate * n))
    if n_out:
        idx = rng.choice(n, size=n_out, replace=False)
        values[idx] *= np.float32(outlier_scale)
    n_zero = int(round(zero_rate * n))
    if n_zero:
        idx = rng.choice(n, size=n_zero, replace=False)
        values[idx] = np.where(rng.integers(0, 2, size=n_zero) == 1, np.float32(-0.0), np.float32(0.0))
    u = values.view(np.uint32).astype(np.uint64)
    bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return bits, rows, cols


def all_cases():
    """name -> (bits, rows, cols) for every golden case."""
    cases = {"float_edge_cases": float_edge_cases()}
    for bits, rows, cols in random_bit_shapes():
        cases[f"random_bits_{rows}x{cols}"] = (bits, rows, cols)
    cases["forced_fallback_tile"] = forced_fallback_tile()
    cases["concentrated_160x2560_s5"] = concentrated(160, 2560, 5)
    cases["concentrated_32x512_s1"] = concentrated(32, 512, 1)
    cases["concentrated_64x512_s1"] = concentrated(64, 512, 1)
    cases["concentrated_32x256_s2"] = concentrated(32, 256, 2)
    cases["gpu_decode_random_64x512"] = gpu_decode_random()
    cases["synthetic_272x2304_s0"] = synthetic_weights(272, 2304, seed=0)
    cases["synthetic_outlier1pct_64x1024_s4"] = synthetic_weights(64, 1024, seed=4, outlier_rate=1e-2, outlier_scale=1024.0)
    return cases
