"""Weight offload (.spec/features/weight-offload: spec.md AC-029, design.md):
the placement rule on CPU against design.md's table; on the GPU, layers
streamed from pinned host memory through the double-buffered staging give
results bit-identical to the same layers resident (same kernels, same
bytes), for SE12 (plain, segmented and fallback tiles) and BF16, across
several tokens; a compressed model with offloaded decoder layers gives the
same logits as without offload."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from se12_b200.offload import place_layers, predicted_stream_ratio


@pytest.mark.parametrize("resident,ratio", [(4, 0.68), (6, 0.63), (10, 0.46), (14, 0.0)])
def test_predicted_ratio_matches_the_design_table(resident, ratio):
    # Gemma 2 9B: T = 18.5 GB BF16, r T = 13.9 GB SE12 (design.md "Why the effect compounds")
    assert predicted_stream_ratio(18.5, 13.9, resident) == pytest.approx(ratio, abs=0.005)


def test_placement_keeps_a_forward_prefix_and_pays_for_staging():
    p = place_layers([10] * 6, 45)  # streaming: 2 x 10 staging, 25 left -> 2 layers resident
    assert p.resident == (0, 1) and p.streamed == (2, 3, 4, 5)
    assert (p.resident_bytes, p.streamed_bytes, p.staging_bytes) == (20, 40, 20)
    assert place_layers([10] * 6, 60).streamed == ()          # everything fits: no staging
    assert place_layers([10] * 6, 19).resident == ()          # less than the staging: all streamed
    assert place_layers([4, 12, 4, 12], 30).resident == (0,)  # staging sized by the largest layer
    with pytest.raises(ValueError):
        place_layers([1, -1], 5)


def test_the_same_rule_streams_fewer_bytes_in_se12():
    bf16 = [156] * 26
    se12 = [117] * 26
    for budget in (500, 1000, 2000):
        b, s = place_layers(bf16, budget), place_layers(se12, budget)
        assert len(s.resident) >= len(b.resident) and s.streamed_bytes < b.streamed_bytes


def _se12_layers(n):
    import bench
    from se12_b200.codec import encode_device
    from se12_b200.device import DeviceSe12Matrix

    dev = torch.device("cuda", 0)
    layers = []
    for i in range(n):
        q = encode_device(bench.synthetic_bf16(torch, 64, 1000, 10 * i, dev))
        k = encode_device(bench.synthetic_bf16(torch, 32, 1000, 10 * i + 1, dev, outlier_rate=1e-2, outlier_scale=1024.0))
        o = encode_device(bench.synthetic_bf16(torch, 1000, 512, 10 * i + 2, dev))
        layers.append([DeviceSe12Matrix.concatenate([q, k]), o])
    assert any(m.fallback_tiles for layer in layers for m in layer)
    return layers


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["se12", "bf16"])
def test_streamed_layers_match_resident_layers_bit_for_bit(fmt):
    from se12_b200.device import bf16_gemv
    from se12_b200.offload import LayerStreamer

    torch.cuda.set_device(0)
    layers = _se12_layers(5)
    if fmt == "bf16":
        layers = [[m.decode() for m in layer] for layer in layers]
    xs = [torch.randn(3, (m.cols if fmt == "se12" else m.shape[1]), device="cuda").to(torch.bfloat16) for m in layers[0]]

    def run(m, x):
        return m.gemv(x) if fmt == "se12" else bf16_gemv(m, x)

    want = [[run(m, x) for m, x in zip(layer, xs)] for layer in layers]
    streamed = [1, 2, 4]  # three streamed layers: an odd cycle, so each alternates staging slots
    streamer = LayerStreamer([layers[i] for i in streamed], "cuda")
    for token in range(3):
        for j, i in enumerate(streamed):
            views = streamer.acquire(j)
            got = [run(m, x) for m, x in zip(views, xs)]
            streamer.release(j)
            for a, b in zip(got, want[i]):
                assert torch.equal(a, b), (token, i)
    with pytest.raises(RuntimeError, match="out of order"):
        streamer.acquire(2)
    torch.cuda.synchronize()


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["exact", "fused"])
def test_offloaded_model_gives_the_same_logits(mode):
    from se12_b200.offload import offload_model
    from se12_b200.runtime import compress_model
    from test_runtime import tiny_gemma

    torch.cuda.set_device(0)
    ref = tiny_gemma().cuda()
    resident = compress_model(copy.deepcopy(ref), mode=mode)
    offloaded = compress_model(copy.deepcopy(ref), mode=mode)
    placement = offload_model(offloaded, budget_bytes=0)
    assert placement.streamed == (0, 1) and placement.resident == ()
    gen = torch.Generator("cuda").manual_seed(5)
    with torch.no_grad():
        for length in (7, 1, 1):  # a prefill, then two decode-sized steps
            ids = torch.randint(0, 1024, (1, length), device="cuda", generator=gen)
            want = resident(ids).logits
            got = offloaded(ids).logits
            assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    torch.cuda.synchronize()
