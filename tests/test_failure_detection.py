"""Failure detection without a GPU fault: a wait on a peer that never writes
runs out, the kernel returns, the status word says so, and the device stays
usable.

One GPU: a peer group of two ranks whose second rank's receive buffer is a
plain local buffer nobody writes (the lost peer). Rank 0's fused GEMV +
all-reduce stores its rows, then waits for rank 1's rows, which never come.
With the wait limit set to 50 ms the kernel gives up, raises the timed-out
bit and leaves y unwritten; after the status is cleared (and the pooled
workspaces zeroed) and the limit restored, ordinary GEMVs on the same
matrix match the fp64 oracle. The same for a chain holding an all-reduced
op. Every wait here is bounded; no test makes a kernel fault or trap.
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

import cases
import se12_oracle as oracle

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-3
SHORT_LIMIT_NS = 50_000_000
DEFAULT_LIMIT_NS = 2_000_000_000


@pytest.fixture(scope="module", autouse=True)
def library():
    from se12_b200 import _build

    _build.build()
    torch.cuda.set_device(0)
    yield


@pytest.fixture()
def short_limit():
    from se12_b200.device import device_status, set_wait_limit_ns, wait_limit_ns

    assert device_status() == 0
    before = wait_limit_ns()
    set_wait_limit_ns(SHORT_LIMIT_NS)
    try:
        yield
    finally:
        torch.cuda.synchronize()
        device_status(clear=True)
        set_wait_limit_ns(before)


class LostPeerGroup:
    """A two-rank peer group on one GPU whose rank 1 never writes."""

    def __init__(self, rows_cap):
        from se12_b200 import _lib

        nbytes = _lib.load().se12_peer_recv_bytes(2, rows_cap)
        self.own = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        self.lost = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")  # stands in for rank 1's buffer
        self.epoch = torch.zeros(4, dtype=torch.int32, device="cuda")
        self.struct = _lib.Se12PeerGroupStruct()
        self.struct.world, self.struct.rank, self.struct.rows_cap = 2, 0, rows_cap
        self.struct.recv[0] = self.own.data_ptr()
        self.struct.recv[1] = self.lost.data_ptr()
        self.struct.epoch = self.epoch.data_ptr()


def matrix_and_input(rows=272, cols=2304, batch=2, seed=3):
    from se12_b200.device import DeviceSe12Matrix

    bits, r, c = cases.synthetic_weights(rows, cols, seed=seed)
    s = oracle.encode(np.asarray(bits, dtype=np.uint16), r, c)

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(dtype)).cuda()

    m = DeviceSe12Matrix(s.rows, s.cols, s.codebook, up(s.sm, np.uint8), up(s.ec, np.uint8), up(s.esc, np.uint8),
                         up(s.fallback_bitmap, np.uint8), up(s.fallback_raw, np.int16))
    xb = oracle.bf16_round(np.random.default_rng(seed).normal(size=(batch, cols)).astype(np.float32))
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
    y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
    return m, x, y64


def assert_usable(m, x, y64):
    from se12_b200.device import device_status

    y = m.gemv(x)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert oracle.max_relative_error(y.cpu().numpy(), y64) <= TOLERANCE


def test_wait_limit_is_settable_and_checked():
    from se12_b200 import _lib
    from se12_b200.device import set_wait_limit_ns, wait_limit_ns

    before = wait_limit_ns()
    assert before == DEFAULT_LIMIT_NS
    try:
        set_wait_limit_ns(123_456_789)
        assert wait_limit_ns() == 123_456_789
        with pytest.raises(_lib.Se12Error):
            set_wait_limit_ns(10)  # below the minimum
    finally:
        set_wait_limit_ns(before)
    assert wait_limit_ns() == before


def test_fused_allreduce_with_a_lost_peer_times_out(short_limit):
    from se12_b200 import _lib
    from se12_b200.device import STATUS_WAIT_TIMEOUT, WORKSPACES, device_status, set_wait_limit_ns, stream_handle

    m, x, y64 = matrix_and_input()
    group = LostPeerGroup(rows_cap=m.rows)
    y = torch.full((x.shape[0], m.rows), float("nan"), device="cuda")
    dev = torch.device("cuda", 0)
    ws = WORKSPACES.get(dev, stream_handle(dev), _lib.load().se12_gemv_workspace_bytes(m.handle, 16))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.call("se12_gemv_allreduce", m.handle, ctypes.c_void_p(x.data_ptr()), x.shape[0], x.stride(0),
              ctypes.c_void_p(y.data_ptr()), y.stride(0), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
              ctypes.byref(group.struct), ctypes.c_void_p(stream_handle(dev)))
    torch.cuda.synchronize()  # the kernel returned: no hang, no CUDA error
    elapsed = time.perf_counter() - t0
    status = device_status(clear=True)
    assert status & STATUS_WAIT_TIMEOUT, status
    assert elapsed < 5.0, elapsed  # one 50 ms limit, not one per waiting value
    assert torch.isnan(y).all()  # no row was written without every rank's part
    set_wait_limit_ns(DEFAULT_LIMIT_NS)
    assert_usable(m, x, y64)


def test_chain_with_a_lost_peer_times_out(short_limit):
    from se12_b200.chain import Se12Chain
    from se12_b200.device import STATUS_WAIT_TIMEOUT, device_status, set_wait_limit_ns

    m, x, y64 = matrix_and_input(rows=1040, cols=2304, batch=1, seed=5)
    m2, x2, y64_2 = matrix_and_input(rows=2048, cols=2304, batch=1, seed=6)
    group = LostPeerGroup(rows_cap=m.rows)
    y = torch.full((1, m.rows), float("nan"), device="cuda")
    y2 = torch.full((1, m2.rows), float("nan"), device="cuda")
    chain = Se12Chain(1)
    chain.add(m2, x2, y2)             # an ordinary op first
    chain.add(m, x, y, peers=group)   # then one all-reduced over the lost peer
    chain.add(m2, x2, y2)             # and one after it
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    chain.run()
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    status = device_status(clear=True)
    assert status & STATUS_WAIT_TIMEOUT, status
    assert elapsed < 5.0, elapsed
    assert torch.isnan(y).all()
    set_wait_limit_ns(DEFAULT_LIMIT_NS)
    chain.reset()
    assert_usable(m, x, y64)
    assert_usable(m2, x2, y64_2)
