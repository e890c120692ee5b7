"""Compressor host logic (CPU): block discovery by the family patterns, the
reference's layer-finding helpers, and the FP8 model assembly it reads."""

import pytest
import torch
import torch.nn as nn


def tiny_qwen3_config(layers=2):
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=layers,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                       max_position_embeddings=256, tie_word_embeddings=False)


def test_find_fp8_blocks_uses_sorted_linear_names():
    from ecf8_b200.compress import find_fp8_blocks
    from ecf8_b200.const import get_fp8_pattern_dict
    from ecf8_b200.fp8_model import fp8_model_from_config
    m = fp8_model_from_config(tiny_qwen3_config(), device="cpu", seed=1)
    blocks = find_fp8_blocks(m, get_fp8_pattern_dict(m.__class__.__name__)["fp8"])
    assert list(blocks) == ["model.layers.0", "model.layers.1"]
    names = [n[len("model.layers.0."):] for n in blocks["model.layers.0"]]
    # one stream per layer, sub-Linears in sorted full-name order (utils.py:188-204)
    assert names == ["mlp.down_proj", "mlp.gate_proj", "mlp.up_proj", "self_attn.k_proj",
                     "self_attn.o_proj", "self_attn.q_proj", "self_attn.v_proj"]


def test_layer_helpers_follow_reference_semantics():
    from ecf8_b200.codec import (find_layers_by_data_type, find_layers_by_layer_type,
                                 find_layers_by_selection, locate_block_by_regex, repo_id_to_model_id)
    m = nn.Sequential(nn.Linear(2, 3), nn.Sequential(nn.Linear(3, 4), nn.ReLU()))
    m[0].weight.data = m[0].weight.data.to(torch.bfloat16)
    assert list(find_layers_by_layer_type(m)) == ["0", "1.0"]
    assert list(find_layers_by_data_type(m, torch.bfloat16)) == ["0"]
    assert list(locate_block_by_regex(m, r"1")) == ["1"]
    # a dotted path is looked up from every module below the start (utils.py:83-117)
    assert list(find_layers_by_selection(m, ["0"])) == ["0", "1.0"]
    assert repo_id_to_model_id("Qwen/Qwen3-8B-FP8") == "models--Qwen--Qwen3-8B-FP8"


def test_fp8_checkpoint_round_trip(tmp_path):
    from ecf8_b200.fp8_model import fp8_model_from_config, load_fp8_checkpoint, save_fp8_checkpoint
    m = fp8_model_from_config(tiny_qwen3_config(), device="cpu", seed=5)
    x = torch.randint(0, 512, (2, 8))
    with torch.no_grad():
        y = m(x).logits
    save_fp8_checkpoint(m, str(tmp_path))
    m2 = load_fp8_checkpoint(str(tmp_path))
    with torch.no_grad():
        assert torch.equal(m2(x).logits, y)


def test_quantize_block128_scales_each_tile():
    from ecf8_b200.fp8_model import quantize_block128
    w = torch.randn(300, 200) * 0.02
    q, s = quantize_block128(w)
    assert q.dtype == torch.float8_e4m3fn and q.shape == (300, 200) and s.shape == (3, 2)
    tile = q[128:256, 0:128].float().abs().max()
    assert tile == 448.0
    deq = q.float() * s.repeat_interleave(128, 0)[:300].repeat_interleave(128, 1)[:, :200]
    assert (deq - w).abs().max() < 0.1 * w.abs().max()


def test_compress_cli_rejects_missing_checkpoint(tmp_path):
    from ecf8_b200.compress import main
    with pytest.raises(SystemExit):
        main(["--repo_id", str(tmp_path / "nope")])


def test_flux_dit_streams_match_reference_pattern_sizes():
    """dit.blocks.N / dit.single_blocks.N streams of the FLUX pattern
    (const.py:30-44): 226,492,416 and 141,557,760 e4m3 weights."""
    from ecf8_b200.compress import find_fp8_blocks
    from ecf8_b200.const import get_fp8_pattern_dict
    from ecf8_b200.dit_model import flux_dit_pipeline
    p = flux_dit_pipeline(device="cpu", seed=0, n_double=1, n_single=1)
    blocks = find_fp8_blocks(p, get_fp8_pattern_dict(p.__class__.__name__)["fp8"])
    sizes = {k: sum(m.weight.numel() for m in v.values()) for k, v in blocks.items()}
    assert sizes == {"dit.blocks.0": 226492416, "dit.single_blocks.0": 141557760}
    assert [n[len("dit.single_blocks.0."):] for n in blocks["dit.single_blocks.0"]] == [
        "norm.linear", "proj_out", "to_qkv_mlp"]
