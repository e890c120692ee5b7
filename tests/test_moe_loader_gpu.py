"""Loader for transformers' fused MoE experts (f2): a Qwen3MoeForCausalLM FP8
checkpoint (per-expert keys on disk, fused 3-D expert parameters in the
installed transformers) is compressed with the reference's qwen3moe pattern
(one stream per attention block and per expert, dfloat/const.py:15-21),
loaded through DFloatModel.from_pretrained, and gives logits identical to the
uncompressed FP8 model; the compressed forward decodes only routed experts."""
import json
import os

import pytest
import torch

from test_moe_loader import tiny_qwen3_moe_config

pytestmark = pytest.mark.gpu


def test_fused_moe_checkpoint_compress_load_identical_logits(cuda_device, tmp_path):
    from ecf8_b200 import DFloatModel
    from ecf8_b200.compress import main
    from ecf8_b200.fp8_model import Fp8FusedExperts, fp8_model_from_config, save_fp8_checkpoint
    from ecf8_b200.run import TensorManager
    model = fp8_model_from_config(tiny_qwen3_moe_config(), device=cuda_device, seed=5)
    x = torch.randint(0, 512, (2, 16), device=cuda_device)
    with torch.no_grad():
        logits = model(x).logits
    ckpt = str(tmp_path / "Qwen3-moe-tiny-FP8")
    save_fp8_checkpoint(model, ckpt)
    save_path = main(["--repo_id", ckpt, "--dfloat_dir", str(tmp_path / "dfloat"), "--save_model",
                      "--validate_cuda", "--model_name", "Qwen/Qwen3-moe-tiny-FP8"])
    pattern = json.load(open(os.path.join(save_path, "pattern_dict.json")))
    assert pattern["fp8"][r"model\.layers\.\d+\.mlp\.experts\.\d+"] == ["down_proj", "gate_proj", "up_proj"]
    assert pattern["fp8"][r"model\.layers\.\d+\.self_attn"] == ["k_proj", "o_proj", "q_proj", "v_proj"]
    from safetensors.torch import load_file
    state = load_file(os.path.join(save_path, "model.safetensors"))
    assert "model.layers.1.mlp.experts.7.encoded" in state  # the reference's per-expert stream keys
    assert "model.layers.1.mlp.experts.7.down_proj.weight_scale_inv" in state
    assert not any(k.endswith("experts.7.down_proj.weight") for k in state)
    TensorManager.clear_device()
    loaded = DFloatModel.from_pretrained(save_path, "DFloat11/Qwen3-moe-tiny-FP8-DF6.5", ckpt, device=cuda_device)
    experts = [m for m in loaded.modules() if isinstance(m, Fp8FusedExperts)]
    assert experts and all(len(m.compressed) == m.num_experts and not m._has_dense() for m in experts)
    decoded = []
    for m in experts:  # record which experts each forward decodes
        orig = m.expert_weights
        m.expert_weights = lambda ex, orig=orig: (decoded.append(list(ex)), orig(ex))[1]
    with torch.no_grad():
        assert torch.equal(loaded(x).logits, logits)
        assert torch.equal(loaded(x).logits, logits)  # overlapped decodes once the tables exist
        one = loaded(x[:1, :1]).logits  # one token: only its top-2 experts per layer
    assert decoded and all(len(d) <= 8 for d in decoded)
    assert all(len(d) == 2 for d in decoded[-len(experts):])
    with torch.no_grad():
        assert torch.equal(one, model(x[:1, :1]).logits)
