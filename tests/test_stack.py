"""GemvStack: a sequence of GEMVs captured once into a CUDA graph and
replayed gives the same bits as the same GEMVs called one by one (the same
kernels and launch configurations; every reduction runs in a fixed order),
also after new inputs are written into the captured buffers."""

import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


def test_graph_replay_matches_direct_calls():
    from se12_b200.codec import encode_device
    from se12_b200.device import bf16_gemv
    from se12_b200.stack import GemvStack

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    mats = []
    # on a 148-SM B200: 8-tile stages, the wide layout, 4-tile stages
    for seed, (rows, cols) in enumerate([(272, 2304), (2304, 9216), (64, 512)]):
        bits, r, c = cases.synthetic_weights(rows, cols, seed=30 + seed)
        w = torch.from_numpy(np.asarray(bits, dtype=np.uint16).view(np.int16).reshape(r, c).copy()).view(torch.bfloat16).to(dev)
        mats.append((encode_device(w), w))
    stack = GemvStack(dev)
    xs, ys = [], []
    for m, _ in mats:
        x = torch.randn(3, m.cols, device=dev).to(torch.bfloat16)
        y = torch.empty(3, m.rows, device=dev)
        stack.add(m, x, y)
        xs.append(x)
        ys.append(y)
    wd = mats[0][1]
    xd = torch.randn(3, wd.shape[1], device=dev).to(torch.bfloat16)
    yd = torch.empty(3, wd.shape[0], device=dev)
    stack.add_dense(wd, xd, yd)
    assert stack.launches == 4
    for step in range(2):
        if step:
            for x in xs + [xd]:
                x.copy_(torch.randn(x.shape, device=dev).to(torch.bfloat16))
        stack.replay()
        torch.cuda.synchronize()
        for (m, _), x, y in zip(mats, xs, ys):
            assert torch.equal(y, m.gemv(x)), f"{m.rows}x{m.cols}, replay {step}"
        assert torch.equal(yd, bf16_gemv(wd, xd)), f"dense, replay {step}"
