"""Compressor end to end on the GPU: an FP8 checkpoint is compressed by
`python -m ecf8_b200.compress`, written in the reference's on-disk layout,
loaded back with DFloatModel.from_pretrained and gives logits identical to
the uncompressed FP8 model."""
import csv
import json
import os

import pytest
import torch

from test_compress import tiny_qwen3_config

pytestmark = pytest.mark.gpu


@pytest.fixture
def fp8_checkpoint(cuda_device, tmp_path):
    from ecf8_b200.fp8_model import fp8_model_from_config, save_fp8_checkpoint
    model = fp8_model_from_config(tiny_qwen3_config(layers=3), device=cuda_device, seed=11)
    x = torch.randint(0, 512, (2, 24), device=cuda_device)
    with torch.no_grad():
        logits = model(x).logits
    path = str(tmp_path / "Qwen3-tiny-FP8")
    save_fp8_checkpoint(model, path)
    return path, x, logits


def test_compress_cli_layout_and_identical_logits(cuda_device, tmp_path, fp8_checkpoint):
    from ecf8_b200 import DFloatModel
    from ecf8_b200.compress import main
    from ecf8_b200.run import TensorManager
    ckpt, x, logits = fp8_checkpoint
    save_path = main(["--repo_id", ckpt, "--dfloat_dir", str(tmp_path / "dfloat"), "--save_model",
                      "--validate_cuda", "--model_name", "Qwen/Qwen3-tiny-FP8"])
    assert save_path.endswith("models--DFloat11--Qwen3-tiny-FP8-DF6.5")
    pattern = json.load(open(os.path.join(save_path, "pattern_dict.json")))
    assert pattern["fp8"] == {r"model\.layers\.\d+": ["mlp.down_proj", "mlp.gate_proj", "mlp.up_proj",
                                                      "self_attn.k_proj", "self_attn.o_proj",
                                                      "self_attn.q_proj", "self_attn.v_proj"]}
    cfg = json.load(open(os.path.join(save_path, "config.json")))
    assert cfg["dfloat_config"]["threads_per_block"] == 512 and cfg["dfloat_config"]["bytes_per_thread"] == 8
    rows = list(csv.DictReader(open(os.path.join(save_path, "entropy.csv"))))
    assert [r["block_name"] for r in rows] == [f"model.layers.{i}" for i in range(3)]
    assert all(0 < float(r["entropy"]) < 4 for r in rows)
    for i in range(3):
        assert os.path.exists(os.path.join(save_path, "cache", f"model.layers.{i}.safetensors"))
    from safetensors.torch import load_file
    state = load_file(os.path.join(save_path, "model.safetensors"))
    assert "model.layers.0.encoded" in state and "model.layers.0.mlp.down_proj.weight" not in state
    assert state["model.layers.0.output_positions"].dtype == torch.uint8

    for original in (ckpt, "Qwen/Qwen3-tiny-FP8"):  # on disk, or only the compressed checkpoint
        TensorManager.clear_device()
        model = DFloatModel.from_pretrained(save_path, "DFloat11/Qwen3-tiny-FP8-DF6.5", original,
                                            device=cuda_device)
        with torch.no_grad():
            assert torch.equal(model(x).logits, logits)


def test_compress_reuses_cached_blocks(cuda_device, tmp_path, fp8_checkpoint):
    from ecf8_b200.compress import main
    ckpt, _, _ = fp8_checkpoint
    args = ["--repo_id", ckpt, "--dfloat_dir", str(tmp_path / "d"), "--model_name", "Qwen/Qwen3-tiny-FP8"]
    save_path = main(args)
    cache = os.path.join(save_path, "cache", "model.layers.0.safetensors")
    stamp = os.path.getmtime(cache)
    main(args + ["--validate_cuda"])
    assert os.path.getmtime(cache) == stamp
