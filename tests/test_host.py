"""Host-side logic of the runtime layer (no GPU)."""
import pytest
import torch
import torch.nn as nn


def test_tensor_manager_grows_and_reuses():
    from ecf8_b200.run import TensorManager
    TensorManager.clear_device() if torch.cuda.is_available() else TensorManager._tensors.clear()
    a = TensorManager.get_tensor("cpu", 100)
    b = TensorManager.get_tensor(torch.device("cpu"), 50)
    assert b.data_ptr() == a.data_ptr() and b.numel() == 50 and b.dtype == torch.float8_e4m3fn
    c = TensorManager.get_tensor("cpu", 200)
    assert c.numel() == 200
    assert TensorManager._tensors[torch.device("cpu")].numel() == 200
    TensorManager._tensors.clear()


def test_dfloat_path_convention():
    from ecf8_b200 import get_dfloat_model_name_or_path
    local, hub = get_dfloat_model_name_or_path("Qwen/Qwen3-8B-FP8", "/d")
    assert local == "/d/models--DFloat11--Qwen3-8B-FP8-DF6.5"
    assert hub == "DFloat11/Qwen3-8B-FP8-DF6.5"


class Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.down = nn.Linear(4, 2, bias=False)
        self.up = nn.Linear(2, 4, bias=False)


def test_inject_weights_splits_in_order():
    from ecf8_b200.run import inject_weights
    blk = Block()
    del blk.down.weight
    del blk.up.weight
    blk.weight_injection_modules = [blk.down, blk.up]
    blk.split_positions = [8]
    flat = torch.arange(16, dtype=torch.float32)
    inject_weights(blk, flat)
    assert blk.down.weight.shape == (2, 4) and blk.down.weight[0, 0] == 0
    assert blk.up.weight.shape == (4, 2) and blk.up.weight[0, 0] == 8
    lin = nn.Linear(3, 2)
    del lin.weight
    inject_weights(lin, torch.arange(6.0))
    assert lin.weight.shape == (2, 3)


def test_process_compressed_tensor_registers_hook_and_drops_weights():
    from ecf8_b200.run import _process_compressed_tensor
    model = nn.Module()
    model.layers = nn.ModuleList([Block()])
    blk = model.layers[0]
    pd = {r"layers\.\d+": ["down", "up"]}
    op = torch.tensor([0, 24], dtype=torch.int64).view(torch.uint8)
    _process_compressed_tensor(blk, "output_positions", op, "layers.0.output_positions", pd, 512, 8)
    assert blk.shared_mem_size == 512 * 4 + 4 + 24
    _process_compressed_tensor(blk, "split_positions", torch.tensor([8]), "layers.0.split_positions",
                               pd, 512, 8)
    assert blk.split_positions == [8]
    _process_compressed_tensor(blk, "encoded", torch.zeros(4, dtype=torch.uint8), "layers.0.encoded",
                               pd, 512, 8)
    assert len(blk._forward_pre_hooks) == 1
    assert blk.weight_injection_modules == [blk.down, blk.up]
    assert "weight" not in blk.down._parameters and "weight" not in blk.up._parameters


def test_decode_launcher_checks_geometry():
    from ecf8_b200.run import _decode
    with pytest.raises(ValueError):
        _decode(grid=(3,), block=(512,), shared_mem=0, args=[1, 1, 1, 1, 1, 1, 3, 4096, 100])
    with pytest.raises(TypeError):
        _decode(grid=(1,), block=(512,), args=[1, 2, 3])


def test_report_model_size():
    from ecf8_b200.run import report_model_size
    m = nn.Sequential(nn.Linear(4, 4, bias=False), nn.Linear(4, 2, bias=False))
    inc, exc, tot = report_model_size(m, [r"^0\."])
    assert abs(inc * 1024 ** 3 - 64) < 1e-6 and abs(exc * 1024 ** 3 - 32) < 1e-6


def test_const_tables_cover_qwen3():
    from ecf8_b200.const import get_default_no_split_pattern, get_fp8_pattern_dict
    assert get_fp8_pattern_dict("Qwen3ForCausalLM")["fp8"] == [r"model\.layers\.\d+"]
    assert get_fp8_pattern_dict("Qwen3MoeForCausalLM")["fp8"][1] == r"model\.layers\.\d+\.mlp\.experts\.\d+"
    assert r"lm_head" in get_default_no_split_pattern("LlamaForCausalLM")
    with pytest.raises(ValueError):
        get_fp8_pattern_dict("GPT2LMHeadModel")


def test_decode_prefetch_chain_stays_out_of_the_module_tree():
    import torch.nn as nn
    from ecf8_b200.run import enable_decode_prefetch, get_hook
    blocks = nn.ModuleList([nn.Linear(2, 2) for _ in range(3)])
    for b in blocks:
        b.register_buffer("encoded", torch.zeros(4, dtype=torch.uint8))
        b.register_buffer("luts", torch.zeros(2, 256, dtype=torch.uint8))
        b.register_forward_pre_hook(get_hook(512, 8))
    keys = list(blocks.state_dict())
    assert enable_decode_prefetch(blocks) == 3
    assert list(blocks.state_dict()) == keys and len(list(blocks.modules())) == 4
    assert blocks[2]._ecf8_next is blocks[0]
    enable_decode_prefetch(blocks, enable=False)
    assert blocks[0]._ecf8_next is None
