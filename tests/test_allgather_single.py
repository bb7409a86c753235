"""Fused GEMV + all-gather (se12_gemv_allgather) on one GPU, with the other
rank's part of the output placed in advance.

A two-rank peer group on one GPU: rank 0's receive buffer and a second
local buffer standing in for rank 1's. Before each call the test writes
rank 1's rows -- tagged with the call's epoch, in the buffer parity the
call reads -- into rank 0's buffer, as rank 1's kernel would have; rank 0's
kernel then finds them there (no kernel waits for another). The whole
output must hold rank 0's GEMV rows (within 1e-3 of the fp64 oracle) and
rank 1's rows bit for bit, and rank 1's buffer must have received rank 0's
rows with the epoch tag. Two calls in a row cover both parities.
"""

from __future__ import annotations

import ctypes

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


class PhantomPair:
    def __init__(self, rows_cap):
        from se12_b200 import _lib

        nbytes = _lib.load().se12_peer_recv_bytes(2, rows_cap)
        self.own = torch.zeros(nbytes // 8, dtype=torch.int64, device="cuda")
        self.other = torch.zeros(nbytes // 8, dtype=torch.int64, device="cuda")
        self.epoch = torch.zeros(4, dtype=torch.int32, device="cuda")
        self.struct = _lib.Se12PeerGroupStruct()
        self.struct.world, self.struct.rank, self.struct.rows_cap = 2, 0, rows_cap
        self.struct.recv[0] = self.own.data_ptr()
        self.struct.recv[1] = self.other.data_ptr()
        self.struct.epoch = self.epoch.data_ptr()


def words(values: np.ndarray, epoch: int) -> np.ndarray:
    bits = values.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((np.uint64(epoch) << np.uint64(32)) | bits).view(np.int64)


@pytest.mark.parametrize("batch", [1, 3])
def test_allgather_with_a_phantom_rank(batch):
    from se12_b200 import _lib
    from se12_b200.device import WORKSPACES, DeviceSe12Matrix, device_status, stream_handle

    rows, cols = 1040, 2304  # 65 tile rows: a ragged last one
    bits, r, c = cases.synthetic_weights(rows, cols, seed=21)
    s = oracle.encode(np.asarray(bits, dtype=np.uint16), r, c)

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(dtype)).cuda()

    m = DeviceSe12Matrix(s.rows, s.cols, s.codebook, up(s.sm, np.uint8), up(s.ec, np.uint8), up(s.esc, np.uint8),
                         up(s.fallback_bitmap, np.uint8), up(s.fallback_raw, np.int16))
    rows_full = 2 * rows
    pair = PhantomPair(rows_cap=rows)
    dev = torch.device("cuda", 0)
    ws = WORKSPACES.get(dev, stream_handle(dev), _lib.load().se12_gemv_workspace_bytes(m.handle, 16))
    rng = np.random.default_rng(batch)
    for call in (1, 2):  # epoch = call, parity = call & 1
        xb = oracle.bf16_round(rng.normal(size=(batch, cols)).astype(np.float32))
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
        theirs = rng.normal(size=(batch, rows)).astype(np.float32)
        base = (call & 1) * 16 * rows_full
        own = pair.own.cpu().numpy()
        for b in range(batch):
            own[base + b * rows_full + rows: base + b * rows_full + 2 * rows] = words(theirs[b], call)
        pair.own.copy_(torch.from_numpy(own))
        y = torch.full((batch, rows_full), float("nan"), device="cuda")
        _lib.call("se12_gemv_allgather", m.handle, ctypes.c_void_p(x.data_ptr()), batch, x.stride(0),
                  ctypes.c_void_p(y.data_ptr()), y.stride(0), 0, rows_full, ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                  ctypes.byref(pair.struct), ctypes.c_void_p(stream_handle(dev)))
        torch.cuda.synchronize()
        assert device_status() == 0
        out = y.cpu().numpy()
        y64 = oracle.gemv_fp64(bits, rows, cols, oracle.bits_to_float32(xb))
        assert oracle.max_relative_error(out[:, :rows], y64) <= TOLERANCE
        assert np.array_equal(out[:, rows:].view(np.uint32), theirs.view(np.uint32))
        # rank 0's rows went to rank 1's buffer, tagged with the epoch
        other = pair.other.cpu().numpy().view(np.uint64)
        for b in range(batch):
            got = other[base + b * rows_full: base + b * rows_full + rows]
            assert np.all((got >> np.uint64(32)) == call)
            assert np.array_equal((got & np.uint64(0xFFFFFFFF)).astype(np.uint32), out[b, :rows].view(np.uint32))
        assert int(pair.epoch[0].item()) == call
