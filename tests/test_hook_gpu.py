"""Decode-before-forward hook end to end: a model whose FP8 blocks are saved
as ECF8 streams, loaded through the loader, gives bit-identical outputs to the
uncompressed model, and all blocks share one per-device scratch buffer."""
import json
import os

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


class FP8Linear(nn.Module):
    """y = x @ (w_fp8 * scale)^T, computed in fp32 (stands in for the model's FP8 matmul)."""

    def __init__(self, i, o, gen, dev):
        super().__init__()
        self.in_features, self.out_features = i, o
        w = torch.randn(o, i, generator=gen, device=dev) * 0.02
        s = 448.0 / w.abs().max()
        self.weight = nn.Parameter((w * s).to(torch.float8_e4m3fn), requires_grad=False)
        self.register_buffer("weight_scale_inv", (1.0 / s).reshape(1))

    def forward(self, x):
        return x @ (self.weight.float() * self.weight_scale_inv).t()


class Block(nn.Module):
    def __init__(self, h, f, gen, dev):
        super().__init__()
        self.down_proj = FP8Linear(f, h, gen, dev)
        self.gate_proj = FP8Linear(h, f, gen, dev)
        self.up_proj = FP8Linear(h, f, gen, dev)

    def forward(self, x):
        return x + self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


class Tiny(nn.Module):
    def __init__(self, dev, seed=0, n=3, h=256, f=512):
        super().__init__()
        g = torch.Generator(device=dev).manual_seed(seed)
        self.layers = nn.ModuleList([Block(h, f, g, dev) for _ in range(n)])

    def forward(self, x):
        for layer in self.layers:
            x = layer(x)
        return x


def save_compressed(model, path):
    """Writes the reference on-disk layout: one safetensors file holding, per
    block, luts / encoded / packed_other_4bits / output_positions (as bytes) /
    gaps / split_positions, plus pattern_dict.json (compress.py:587-680)."""
    from safetensors.torch import save_file
    from ecf8_b200.codec import compress_fp8
    tensors = {}
    names = ["down_proj", "gate_proj", "up_proj"]
    for i, blk in enumerate(model.layers):
        ws = [getattr(blk, n).weight.data.reshape(-1) for n in names]
        flat = torch.cat(ws)
        c = compress_fp8(flat)
        pre = f"layers.{i}."
        tensors[pre + "luts"] = c["luts"].cpu()
        tensors[pre + "encoded"] = c["encoded"].cpu()
        tensors[pre + "packed_other_4bits"] = c["packed_other_4bits"].cpu()
        tensors[pre + "output_positions"] = c["output_positions"].view(torch.uint8).cpu()
        tensors[pre + "gaps"] = c["gaps"].cpu()
        tensors[pre + "split_positions"] = torch.cumsum(torch.tensor([w.numel() for w in ws]), 0)[:-1]
        for n in names:
            tensors[pre + n + ".weight_scale_inv"] = getattr(blk, n).weight_scale_inv.cpu()
    save_file(tensors, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "pattern_dict.json"), "w") as f:
        json.dump({"fp8": {r"layers\.\d+": names}, "bf16": {}}, f)


@pytest.mark.parametrize("parallel", [False, True])
def test_hooked_model_matches_uncompressed(cuda_device, tmp_path, parallel):
    from ecf8_b200 import load_and_replace_tensors, load_and_replace_tensors_parallel
    from ecf8_b200.run import TensorManager
    dev = cuda_device
    ref = Tiny(dev)
    x = torch.randn(8, 256, device=dev)
    y_ref = ref(x)
    save_compressed(ref, str(tmp_path))
    model = Tiny(dev, seed=123)  # different weights: must be replaced by the streams
    cfg = {"threads_per_block": 512, "bytes_per_thread": 8,
           "pattern_dict": json.load(open(tmp_path / "pattern_dict.json"))}
    loader = load_and_replace_tensors_parallel if parallel else load_and_replace_tensors
    loader(model, str(tmp_path), cfg)
    for blk in model.layers:
        assert "weight" not in blk.down_proj._parameters
    model.to(dev)
    TensorManager.clear_device()
    y = model(x)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    # Later forwards decode with the tables built on the first one, each
    # launch overlapping the previous kernel (ECF8_DECODE_OVERLAP_PREVIOUS).
    for _ in range(3):
        assert torch.equal(model(x), y_ref)
    # every block decoded into the same per-device scratch
    ptrs = {blk.down_proj.weight.data_ptr() for blk in model.layers}
    assert len(ptrs) == 1
    assert TensorManager._tensors[dev].numel() == 3 * 256 * 512


def test_hooked_model_through_the_dfloat_import_path(cuda_device, tmp_path):
    """The same round trip with the reference's import path only
    (``from dfloat.run import ...``, ``from dfloat.run.run import TensorManager``)."""
    from dfloat.run import load_and_replace_tensors_parallel
    from dfloat.run.run import TensorManager
    dev = cuda_device
    ref = Tiny(dev)
    x = torch.randn(8, 256, device=dev)
    y_ref = ref(x)
    save_compressed(ref, str(tmp_path))
    model = Tiny(dev, seed=7)
    cfg = {"threads_per_block": 512, "bytes_per_thread": 8,
           "pattern_dict": json.load(open(tmp_path / "pattern_dict.json"))}
    load_and_replace_tensors_parallel(model, str(tmp_path), cfg)
    model.to(dev)
    TensorManager.clear_device()
    for _ in range(3):
        assert torch.equal(model(x), y_ref)


def test_reference_launcher_caches_tables_and_survives_reused_lut_memory(cuda_device):
    """`_decode` with the reference's call convention (compress.py:109-124):
    the first call on a LUT address builds a table, later calls reuse it; new
    LUTs written to the same address are detected by the kernel, so the decode
    stays exact, and clear_cache() drops the tables."""
    import numpy as np
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__)))
    from conftest import load_golden
    from helpers import to_device
    from dfloat.run import _decode
    a, b = load_golden("gauss_per_tensor"), load_golden("fibonacci_depth16")
    luts = torch.zeros(18, 256, dtype=torch.uint8, device=cuda_device)

    def run(s):
        d = to_device(s, cuda_device)
        n_l = s["luts"].shape[0]
        luts[:n_l] = d["luts"]
        n = s["fp8"].size
        out = torch.zeros(n, dtype=torch.uint8, device=cuda_device)
        grid = (-(-d["encoded"].numel() // 4096),)
        _decode(grid=grid, block=(512,), shared_mem=0,
                args=[luts.data_ptr(), d["encoded"].data_ptr(), d["packed_other_4bits"].data_ptr(),
                      d["output_positions"].data_ptr(), d["gaps"].data_ptr(), out.data_ptr(), n_l,
                      d["encoded"].numel(), n])
        torch.cuda.synchronize()
        return np.array_equal(out.cpu().numpy(), s["fp8"])

    _decode.clear_cache()
    assert run(a) and run(a)
    assert len(_decode._tables) == 1
    assert run(b)  # other LUTs at the same address (same n_luts or not): still exact
    assert run(a)
    _decode.clear_cache()
    assert not _decode._tables


def test_decode_prefetch_mode_matches_uncompressed(cuda_device, tmp_path):
    """enable_decode_prefetch: each block's hook decodes the next block on a
    side stream into the second scratch buffer; outputs stay bit-identical
    over repeated forwards (also with the side-stream decodes limited to a
    few CTAs), and switching from the plain hook and back to it re-points the
    weights each time."""
    from ecf8_b200 import enable_decode_prefetch, load_and_replace_tensors
    from ecf8_b200.run import TensorManager
    dev = cuda_device
    ref = Tiny(dev, n=4)
    x = torch.randn(8, 256, device=dev)
    y_ref = ref(x)
    save_compressed(ref, str(tmp_path))
    model = Tiny(dev, seed=9, n=4)
    cfg = {"threads_per_block": 512, "bytes_per_thread": 8,
           "pattern_dict": json.load(open(tmp_path / "pattern_dict.json"))}
    load_and_replace_tensors(model, str(tmp_path), cfg)
    model.to(dev)
    TensorManager.clear_device()
    keys = list(model.state_dict())
    assert torch.equal(model(x), y_ref)  # plain hook first: plain -> prefetch -> plain below
    assert torch.equal(model(x), y_ref)
    assert enable_decode_prefetch(model) == 4
    assert list(model.state_dict()) == keys  # the block chain is not part of the module tree
    for _ in range(4):
        assert torch.equal(model(x), y_ref)
    # the blocks alternate between two buffers
    ptrs = [blk.down_proj.weight.data_ptr() for blk in model.layers]
    assert len(set(ptrs)) == 2
    # side-stream decodes limited to a few CTAs: the same bytes
    assert enable_decode_prefetch(model, ctas=5) == 4
    for _ in range(3):
        assert torch.equal(model(x), y_ref)
    enable_decode_prefetch(model, enable=False)
    assert torch.equal(model(x), y_ref)
