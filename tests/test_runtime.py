"""Drop-in compressed layers (model-integration, .spec/features/
model-integration/spec.md AC-015, AC-016, AC-025) on a small random-init
Gemma-2 built from its config (no checkpoint download).

* "exact" mode: logits identical bit for bit to the uncompressed model;
* "fused" mode: logits within a small tolerance, same greedy tokens;
* packed round trip: pack the model's safetensors with the GPU packer, load
  into a fresh skeleton, exact logits identical to the original's;
* weight memory: the compressed model's weights take <= 80 % of the original's.
"""

from __future__ import annotations

import copy

import pytest
import torch


def test_mode_is_validated():
    from se12_b200.runtime import _check_mode

    with pytest.raises(ValueError):
        _check_mode("turbo")


def test_only_bf16_layers_are_eligible():
    from se12_b200.runtime import CompressedLinear

    with pytest.raises(TypeError):
        CompressedLinear.from_linear(torch.nn.Linear(16, 16))  # fp32: refused before any GPU work


def tiny_gemma(seed: int = 0):
    from transformers import Gemma2Config, Gemma2ForCausalLM

    cfg = Gemma2Config(vocab_size=1024, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=2, num_key_value_heads=1, head_dim=128, max_position_embeddings=256,
                       attn_implementation="eager")
    torch.manual_seed(seed)
    return Gemma2ForCausalLM(cfg).to(torch.bfloat16).eval()


def weight_bytes(model) -> int:
    from se12_b200.runtime import CompressedEmbedding, CompressedLinear

    seen, total = set(), 0
    for mod in model.modules():
        if isinstance(mod, (CompressedLinear, CompressedEmbedding)) and id(mod.matrix) not in seen:
            seen.add(id(mod.matrix))
            total += mod.matrix.byte_size
    ptrs = set()
    for t in list(model.parameters()) + [b for b in model.buffers() if b is not None]:
        if t.data_ptr() not in ptrs:
            ptrs.add(t.data_ptr())
            total += t.numel() * t.element_size()
    return total


@pytest.mark.gpu
def test_exact_mode_logits_are_bit_identical():
    from se12_b200.runtime import CompressedEmbedding, CompressedLinear, compress_model

    ref = tiny_gemma().cuda()
    ids = torch.randint(0, 1024, (2, 12), device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    with torch.no_grad():
        want = ref(ids).logits
        packed = compress_model(copy.deepcopy(ref), mode="exact")
        got = packed(ids).logits
    assert all(not isinstance(m, torch.nn.Linear) for m in packed.modules()
               if not isinstance(m, (CompressedLinear, CompressedEmbedding)))
    assert isinstance(packed.lm_head, CompressedLinear) and isinstance(packed.model.embed_tokens, CompressedEmbedding)
    assert packed.lm_head.matrix is packed.model.embed_tokens.matrix  # tied weights share one set of streams
    assert torch.equal(got.view(torch.int16) if got.dtype == torch.bfloat16 else got, want.view(torch.int16) if want.dtype == torch.bfloat16 else want)
    assert weight_bytes(packed) <= 0.80 * weight_bytes(ref)


@pytest.mark.gpu
def test_fused_mode_matches_within_tolerance():
    from se12_b200.runtime import compress_model

    ref = tiny_gemma().cuda()
    ids = torch.randint(0, 1024, (1, 1), device="cuda", generator=torch.Generator("cuda").manual_seed(2))
    with torch.no_grad():
        want = ref(ids).logits.float()
        got = compress_model(copy.deepcopy(ref), mode="fused")(ids).logits.float()
    err = ((got - want).abs() / want.abs().clamp_min(1.0)).max().item()
    assert err <= 2e-2, err
    assert torch.equal(got.argmax(-1), want.argmax(-1))


@pytest.mark.gpu
def test_packed_round_trip_into_fresh_model(tmp_path):
    import safetensors.torch

    from se12_b200.packed import pack_model
    from se12_b200.runtime import load_packed

    ref = tiny_gemma(seed=0)
    state = {k: v.contiguous() for k, v in ref.state_dict().items() if k != "lm_head.weight"}  # tied: saved once
    (tmp_path / "model").mkdir()
    safetensors.torch.save_file(state, str(tmp_path / "model" / "model.safetensors"))
    summary = pack_model(tmp_path / "model", tmp_path / "packed")
    assert summary.encoded == 1 + 7 * 2  # embedding + 7 projections per layer
    fresh = load_packed(tmp_path / "packed", tiny_gemma(seed=123), mode="exact")
    ids = torch.randint(0, 1024, (1, 9), device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    with torch.no_grad():
        want = ref.cuda()(ids).logits
        got = fresh(ids).logits
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.gpu
def test_grouped_projections_run_one_gemv_per_group():
    """q/k/v and gate/up become one segmented matrix each; a block's
    projections of one input run one fused GEMV, and the logits match both
    the ungrouped fused model and the original within the fused tolerance."""
    from se12_b200.runtime import ProjectionGroup, compress_model

    ref = tiny_gemma().cuda()
    ids = torch.randint(0, 1024, (1, 1), device="cuda", generator=torch.Generator("cuda").manual_seed(4))
    grouped = compress_model(copy.deepcopy(ref), mode="fused")
    plain = compress_model(copy.deepcopy(ref), mode="fused", group=False)
    attn, mlp = grouped.model.layers[0].self_attn, grouped.model.layers[0].mlp
    assert attn.q_proj.group is attn.k_proj.group is attn.v_proj.group is not None
    assert mlp.gate_proj.group is mlp.up_proj.group is not None and mlp.down_proj.group is None
    assert len(attn.q_proj.matrix.segments) == 3
    for name in ("q_proj", "k_proj", "v_proj"):  # each member's rows decode to its own weight
        want = getattr(ref.model.layers[0].self_attn, name).weight
        assert torch.equal(getattr(attn, name).weight_bf16().view(torch.int16), want.view(torch.int16))

    calls = []
    for mod in grouped.modules():
        if isinstance(getattr(mod, "group", None), ProjectionGroup) and mod.group not in calls:
            group, gemv = mod.group, mod.group.matrix.gemv
            group.matrix.gemv = lambda x, out=None, _g=gemv: (calls.append(1), _g(x, out))[1]
            calls.append(group)
    groups = sum(1 for c in calls if c != 1)
    del calls[:]
    with torch.no_grad():
        want = ref(ids).logits.float()
        got = grouped(ids).logits.float()
        base = plain(ids).logits.float()
    assert len(calls) == groups == 2 * 2  # two layers x (qkv, gate_up), one GEMV each
    for other in (want, base):
        err = ((got - other).abs() / other.abs().clamp_min(1.0)).max().item()
        assert err <= 2e-2, err
    assert torch.equal(got.argmax(-1), want.argmax(-1))


@pytest.mark.gpu
def test_projection_group_recomputes_for_a_new_input():
    from se12_b200.runtime import compress_model

    model = compress_model(tiny_gemma().cuda(), mode="fused")
    attn = model.model.layers[0].self_attn
    x1 = torch.randn(1, 256, device="cuda").to(torch.bfloat16)
    x2 = torch.randn(1, 256, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        q1 = attn.q_proj(x1)
        k2 = attn.k_proj(x2)  # another input: not the cached result
        k2_alone = attn.k_proj(x2)
        x1.mul_(2)  # same storage, new version
        q1b = attn.q_proj(x1)
    assert torch.equal(k2, k2_alone)
    assert not torch.equal(q1, q1b)
    assert torch.allclose(q1b.float(), 2 * q1.float(), rtol=1e-2, atol=1e-2)
