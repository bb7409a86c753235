"""The decoder shapes the bench and the tensor-parallel step use: weight
counts of the benchmark configurations (Gemma-2 2B / 9B / 27B, Llama-3.1
70B), and the tile alignment that lets shards be cut from the packed
streams without re-encoding (rows split on multiples of 16, columns on
multiples of 256)."""

import pytest

from se12_b200.shapes import CONFIGS


@pytest.mark.parametrize("name,per_layer,total", [
    ("gemma2-2b", 77.86e6, 2.614e9),     # lm_head 256000 x 2304 included
    ("gemma2-9b", 198.2e6, 8.32e9 + 0.92e9),
    ("gemma2-27b", 566.2e6, 27.23e9),
    ("llama3.1-70b", 855.6e6, 69.50e9),
])
def test_weight_counts(name, per_layer, total):
    s = CONFIGS[name]
    assert s.weights_per_layer == pytest.approx(per_layer, rel=1e-3)
    assert s.total_weights == pytest.approx(total, rel=2e-3)


def test_gemma2_2b_step_is_the_bench_workload():
    s = CONFIGS["gemma2-2b"]
    shapes = {name: (rows, cols) for name, rows, cols, _ in s.layer_matrices()}
    assert shapes == {"q_proj": (2048, 2304), "k_proj": (1024, 2304), "v_proj": (1024, 2304), "o_proj": (2304, 2048),
                      "gate_proj": (9216, 2304), "up_proj": (9216, 2304), "down_proj": (2304, 9216)}
    assert s.lm_head()[1:3] == (256000, 2304) and s.layers == 26
    assert s.total_weights == 2614099968
    # the grouped projections multiply the same input
    kinds = {name: kind for name, _, _, kind in s.layer_matrices()}
    for _, members in s.GROUPS:
        assert len({kinds[m] for m in members}) == 1


@pytest.mark.parametrize("name", sorted(CONFIGS))
@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_tensor_parallel_shards_fall_on_tile_edges(name, ranks):
    """Megatron split (q/k/v/gate/up and the LM head by output rows, o and
    down by input columns) as sharding.py cuts it: contiguous ranges that
    start on tile edges, cover the matrix, and differ by at most one tile;
    equal shards for the survey's tensor-parallel configurations (27B and
    70B on up to 8 GPUs)."""
    from se12_b200.sharding import col_range, row_range

    s = CONFIGS[name]
    mats = [(m, r, c, m in ("o_proj", "down_proj")) for m, r, c, _ in s.layer_matrices()]
    mats.append(("lm_head", s.vocab, s.hidden, False))
    for mat, rows, cols, by_cols in mats:
        n, unit = (cols, 256) if by_cols else (rows, 16)
        ranges = [(col_range if by_cols else row_range)(n, ranks, r) for r in range(ranks)]
        assert ranges[0][0] == 0 and ranges[-1][1] == n, (mat, ranges)
        assert all(a[1] == b[0] and a[0] % unit == 0 for a, b in zip(ranges, ranges[1:])), (mat, ranges)
        tiles = [-(-(stop - start) // unit) for start, stop in ranges]
        assert max(tiles) - min(tiles) <= 1, (mat, tiles)
        if name in ("gemma2-27b", "llama3.1-70b"):
            assert len({stop - start for start, stop in ranges}) == 1, (mat, ranges)
