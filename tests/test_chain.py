"""Chains (se12_chain_*: a sequence of GEMVs in one persistent launch)
through the C ABI, against the fp64 oracle.

Every op's y must satisfy max |y - y64| / max(|y64|, 1) <= 1e-3 (the GEMV
tolerance of the single-call tests), for chains that mix shapes which reach
every code path of the chain kernel: rows shared by the warps of a CTA and rows split between CTAs,
rows held by one warp, padded rows and columns (K % 256 != 0, K % 8 != 0),
segmented matrices (one codebook per segment), escape-heavy and fallback
tiles, a codebook whose padding weight is +inf, column-split ops (x too
large for shared memory at batch 16) and the dense BF16 variant. Results
are bit-identical across launches and under CUDA-graph replay.
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


def weights(kind, rows, cols, seed):
    if kind == "synthetic":
        return cases.synthetic_weights(rows, cols, seed=seed)
    if kind == "outliers":  # 1 % outliers x1024: most tiles fall back
        return cases.synthetic_weights(rows, cols, seed=seed, outlier_rate=1e-2, outlier_scale=1024.0)
    if kind == "escapes":   # 0.2 % outliers: many escapes, few fallback tiles
        return cases.synthetic_weights(rows, cols, seed=seed, outlier_rate=2e-3, outlier_scale=512.0)
    if kind == "concentrated":
        return cases.concentrated(rows, cols, seed=seed)
    raise ValueError(kind)


# (kind, rows, cols): shapes of every size class, in chain order
CHAIN = [
    ("synthetic", 2048, 2304),   # q-like: rows split over a few warps
    ("synthetic", 2304, 2048),   # o-like
    ("escapes", 1024, 2304),
    ("synthetic", 33, 300),      # padded rows and columns, K % 8 != 0
    ("outliers", 160, 2560),     # fallback tiles
    ("synthetic", 2304, 9216),   # down-like: rows split between CTAs
    ("synthetic", 16, 65536),    # one tile row split between CTAs (an even split of the tiles)
    ("escapes", 48, 32768),      # three tile rows, each split between several CTAs
    ("concentrated", 160, 2560),
    ("synthetic", 1, 1),
    ("synthetic", 9216, 2304),   # gate-like: rows held by one warp
]

_mats: dict = {}


def fixture(kind, rows, cols):
    key = (kind, rows, cols)
    if key not in _mats:
        bits, r, c = weights(kind, rows, cols, seed=rows * 3 + cols)
        _mats[key] = (bits, device_matrix(oracle.encode(bits, r, c)))
    return _mats[key]


def bf16_input(batch, cols, seed, ldx=None):
    xb = oracle.bf16_round(np.random.default_rng(seed).normal(0.0, 1.0, size=(batch, cols)).astype(np.float32))
    ld = ldx or (cols + 7) // 8 * 8
    x = torch.full((batch, ld), float("nan"), dtype=torch.bfloat16, device="cuda")  # columns past K: anything
    x[:, :cols] = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    return xb, x


def build_chain(batch, specs, seed=0):
    from se12_b200.chain import Se12Chain

    chain = Se12Chain(batch)
    entries = []
    for n, (kind, rows, cols) in enumerate(specs):
        bits, m = fixture(kind, rows, cols)
        xb, x = bf16_input(batch, cols, seed=seed + 7 * n + batch)
        y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
        chain.add(m, x, y)
        entries.append((bits, rows, cols, xb, y))
    return chain, entries


def check(entries):
    for bits, rows, cols, xb, y in entries:
        y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
        err = oracle.max_relative_error(y.cpu().numpy(), y64)
        assert err <= TOLERANCE, f"{rows}x{cols}: max rel err {err:.3e}"


@pytest.mark.parametrize("batch", [1, 2, 3, 4, 8, 9, 16])
def test_chain_matches_fp64_oracle(batch):
    from se12_b200.device import device_status

    chain, entries = build_chain(batch, CHAIN)
    chain.run()
    torch.cuda.synchronize()
    assert device_status() == 0
    check(entries)
    info = chain.info()
    assert info["grid"] == torch.cuda.get_device_properties(0).multi_processor_count
    assert info["gemvs"] == len(CHAIN) and info["ops"] >= len(CHAIN)


def test_chain_is_deterministic_across_launches():
    chain, entries = build_chain(4, CHAIN)
    chain.run()
    first = [e[4].clone() for e in entries]
    for _ in range(3):
        for e in entries:
            e[4].fill_(float("nan"))
        chain.run()
        for f, e in zip(first, entries):
            assert torch.equal(f, e[4])


def test_chain_graph_replay_and_new_inputs():
    chain, entries = build_chain(2, CHAIN[:4], seed=11)
    chain.run()  # first launch outside the capture (uploads the descriptors)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        chain.run()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    check(entries)
    # new inputs written into the captured buffers
    fresh = []
    for n, (bits, rows, cols, _, y) in enumerate(entries):
        xb, x = bf16_input(2, cols, seed=100 + n)
        chain._keep[4 * n + 2][:, :cols].copy_(x[:, :cols])
        fresh.append((bits, rows, cols, xb, y))
    graph.replay()
    torch.cuda.synchronize()
    check(fresh)
    del graph


def test_chain_splits_columns_when_x_does_not_fit():
    """At batch 16, x of a 9216-column matrix (295 KB) exceeds shared
    memory: the GEMV runs as column blocks that accumulate into y."""
    chain, entries = build_chain(16, [("synthetic", 2304, 9216), ("synthetic", 272, 2304)])
    assert chain.ops > chain.gemvs
    chain.run()
    torch.cuda.synchronize()
    check(entries)


def test_chain_later_op_overwrites_earlier_output():
    """Ops run in order: two GEMVs writing one y leave the second's rows."""
    from se12_b200.chain import Se12Chain

    b1, m1 = fixture("synthetic", 2048, 2304)
    b2, m2 = fixture("escapes", 1024, 2304)
    x1b, x1 = bf16_input(1, 2304, seed=1)
    x2b, x2 = bf16_input(1, 2304, seed=2)
    y = torch.zeros(1, 2048, dtype=torch.float32, device="cuda")
    chain = Se12Chain(1)
    chain.add(m1, x1, y)
    chain.add(m2, x2, y)
    for _ in range(2):
        chain.run()
        torch.cuda.synchronize()
        out = y.cpu().numpy()
        assert oracle.max_relative_error(out[:, :1024], oracle.gemv_fp64(b2, 1024, 2304, oracle.bits_to_float32(x2b))) <= TOLERANCE
        assert oracle.max_relative_error(out[:, 1024:], oracle.gemv_fp64(b1, 2048, 2304, oracle.bits_to_float32(x1b))[:, 1024:]) <= TOLERANCE


def test_chain_segmented_matrix():
    from se12_b200.chain import Se12Chain
    from se12_b200.device import DeviceSe12Matrix

    parts = [fixture("synthetic", 2048, 2304), fixture("escapes", 1024, 2304), fixture("concentrated", 160, 2560)]
    m = DeviceSe12Matrix.concatenate([parts[0][1], parts[1][1]])
    bits = np.concatenate([parts[0][0], parts[1][0]])
    xb, x = bf16_input(3, 2304, seed=5)
    y = torch.empty(3, m.rows, dtype=torch.float32, device="cuda")
    chain = Se12Chain(3)
    chain.add(m, x, y)
    chain.run()
    torch.cuda.synchronize()
    err = oracle.max_relative_error(y.cpu().numpy(), oracle.gemv_fp64(bits, m.rows, 2304, oracle.bits_to_float32(xb)))
    assert err <= TOLERANCE


def test_chain_infinite_padding_weight():
    """codebook[0] == 255 with K % 256 != 0: the padding weights would decode
    to +inf; the finite rows must still match the oracle."""
    from se12_b200.chain import Se12Chain

    rows, cols = 64, 300
    w = np.random.default_rng(9).normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
    w[:40, :] = np.inf
    bits = oracle.bf16_round(w).reshape(-1)
    streams = oracle.encode(bits, rows, cols)
    assert streams.codebook[0] == 255
    m = device_matrix(streams)
    xb = oracle.bf16_round(np.abs(np.random.default_rng(2).normal(0.0, 1.0, size=(2, cols))) + 0.01)
    x = torch.zeros(2, 304, dtype=torch.bfloat16, device="cuda")
    x[:, :cols] = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y = torch.empty(2, rows, dtype=torch.float32, device="cuda")
    chain = Se12Chain(2)
    chain.add(m, x, y)
    chain.run()
    torch.cuda.synchronize()
    out = y.cpu().numpy()
    y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
    assert np.isposinf(out[:, :40]).all()
    assert oracle.max_relative_error(out[:, 40:], y64[:, 40:]) <= TOLERANCE


@pytest.mark.parametrize("batch", [1, 8, 16])
def test_dense_chain_matches_fp64(batch):
    from se12_b200.chain import Se12Chain

    chain = Se12Chain(batch, dense=True)
    entries = []
    for n, (rows, cols) in enumerate([(2304, 9216), (33, 300), (256, 2304), (9216, 2304)]):
        bits, _, _ = cases.synthetic_weights(rows, cols, seed=11 + n)
        w = torch.from_numpy(np.asarray(bits, dtype=np.uint16).view(np.int16).reshape(rows, cols)).view(torch.bfloat16).cuda()
        if cols % 8:
            wp = torch.zeros(rows, (cols + 7) // 8 * 8, dtype=torch.bfloat16, device="cuda")
            wp[:, :cols] = w
            w = wp[:, :cols]
        xb, x = bf16_input(batch, cols, seed=n)
        y = torch.empty(batch, rows, dtype=torch.float32, device="cuda")
        chain.add_dense(w, x, y)
        entries.append((bits, rows, cols, xb, y))
    chain.run()
    torch.cuda.synchronize()
    check(entries)


def test_gemv_stack_chain_mode_matches_launch_per_gemv():
    """GemvStack(chain=True) runs the same sequence as one launch: every
    output within the tolerance of the launch-per-GEMV stack's."""
    from se12_b200.stack import GemvStack

    outs = {}
    for mode in (False, True):
        st = GemvStack("cuda", chain=mode)
        ys = []
        for n, (kind, rows, cols) in enumerate(CHAIN[:6]):
            _, m = fixture(kind, rows, cols)
            _, x = bf16_input(1, cols, seed=n)
            y = torch.empty(1, rows, dtype=torch.float32, device="cuda")
            st.add(m, x[:, :cols], y)
            ys.append(y)
        st.replay()
        torch.cuda.synchronize()
        outs[mode] = ys
        assert st.launches == (1 if mode else 6)
    for a, b in zip(outs[False], outs[True]):
        err = float(((a.double() - b.double()).abs() / a.double().abs().clamp_min(1.0)).max())
        assert err <= TOLERANCE
