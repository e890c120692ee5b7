"""Fused MoE experts on CPU: the per-expert checkpoint layout of
Fp8FusedExperts, block discovery for the reference's qwen3moe pattern, and
the loader's routing of per-expert keys into the fused parameters."""
import pytest
import torch


def tiny_qwen3_moe_config(layers=2):
    from transformers import Qwen3MoeConfig
    return Qwen3MoeConfig(vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
                          num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                          num_experts=8, num_experts_per_tok=2, decoder_sparse_step=1, mlp_only_layers=[],
                          norm_topk_prob=True, tie_word_embeddings=False, max_position_embeddings=128)


def test_fused_experts_state_dict_uses_per_expert_keys_and_round_trips():
    from ecf8_b200.fp8_model import Fp8FusedExperts, fp8_model_from_config
    model = fp8_model_from_config(tiny_qwen3_moe_config(), device="cpu", seed=3)
    fused = [m for m in model.modules() if isinstance(m, Fp8FusedExperts)]
    assert len(fused) == 2 and fused[0].num_experts == 8
    state = model.state_dict()
    assert state["model.layers.0.mlp.experts.3.gate_proj.weight"].shape == (128, 256)
    assert state["model.layers.0.mlp.experts.3.down_proj.weight"].shape == (256, 128)
    assert state["model.layers.0.mlp.experts.3.up_proj.weight_scale_inv"].shape == (1, 2)
    assert not any("gate_up_proj" in k for k in state)
    other = fp8_model_from_config(tiny_qwen3_moe_config(), device="cpu", seed=None)
    from ecf8_b200.run import _load_one
    params, buffers, keys = dict(other.named_parameters()), dict(other.named_buffers()), set(other.state_dict())
    for k, v in state.items():
        _load_one(other, k, v.clone(), params, buffers, keys, {}, 512, 8)
    got = other.state_dict()
    for k, v in state.items():
        assert torch.equal(got[k].view(torch.uint8) if v.dtype == torch.float8_e4m3fn else got[k],
                           v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else v), k


def test_compressor_finds_one_block_per_expert():
    from ecf8_b200.compress import find_fp8_blocks
    from ecf8_b200.const import get_fp8_pattern_dict
    from ecf8_b200.fp8_model import fp8_model_from_config
    model = fp8_model_from_config(tiny_qwen3_moe_config(), device="cpu", seed=3)
    blocks = find_fp8_blocks(model, get_fp8_pattern_dict("Qwen3MoeForCausalLM")["fp8"])
    experts = sorted(b for b in blocks if ".experts." in b)
    assert len(experts) == 16 and "model.layers.1.mlp.experts.7" in experts
    assert list(blocks["model.layers.0.mlp.experts.2"]) == [
        "model.layers.0.mlp.experts.2.down_proj", "model.layers.0.mlp.experts.2.gate_proj",
        "model.layers.0.mlp.experts.2.up_proj"]
    assert list(blocks["model.layers.0.self_attn"]) == [
        f"model.layers.0.self_attn.{p}_proj" for p in ("k", "o", "q", "v")]
    sd = model.state_dict()
    lay = blocks["model.layers.0.mlp.experts.2"]
    assert torch.equal(lay["model.layers.0.mlp.experts.2.gate_proj"].weight.view(torch.uint8),
                       sd["model.layers.0.mlp.experts.2.gate_proj.weight"].view(torch.uint8))


def test_expert_stream_split_positions_are_checked():
    from ecf8_b200.fp8_model import Fp8FusedExperts
    m = Fp8FusedExperts(2, 256, 128, torch.nn.functional.silu)
    m.add_expert_stream(0, "split_positions", torch.tensor([256 * 128, 2 * 256 * 128]))
    with pytest.raises(ValueError):
        m.add_expert_stream(0, "split_positions", torch.tensor([128, 256]))


def test_partly_compressed_experts_keep_their_dense_weights():
    """Streams for some experts only: the dense parameters stay (needed by
    the others) and every expert's weights come from the right place."""
    from ecf8_b200.fp8_model import Fp8FusedExperts
    m = Fp8FusedExperts(4, 256, 128, torch.nn.functional.silu)
    for k in ("luts", "packed_other_4bits", "output_positions", "gaps"):
        m.add_expert_stream(1, k, torch.zeros(4, dtype=torch.uint8))
    m.add_expert_stream(1, "encoded", torch.zeros(4, dtype=torch.uint8))
    assert m.compressed == {1} and m._has_dense()
    w = m.expert_weights([0, 2])
    assert w[0][0].data_ptr() == m.gate_up_proj[0].data_ptr() and w[1][1].shape == (256, 128)
