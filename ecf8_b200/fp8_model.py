"""FP8 (e4m3, 128x128 block-scaled) Linear layers and model assembly.

The reference compressor and loader take their FP8 models from transformers
(`AutoModelForCausalLM.from_pretrained` of an FP8 checkpoint, whose Linear
layers become `FP8Linear`, scripts/compress.py:495-498, run.py:483-566).
That route needs accelerate and hub-loaded matmul kernels, neither of which
this environment has, so this module builds the same model shape itself:

* `Fp8Linear`: weight e4m3 [out, in] + `weight_scale_inv` f32 [ceil(out/128),
  ceil(in/128)], the layout of FP8 checkpoints such as Qwen3-8B-FP8.  Its
  forward is a block-scaled FP8 GEMM that reads the e4m3 weight directly
  (activations quantized per 1x128 group, weights scaled per 128x128 tile,
  the scheme of transformers' FP8Linear), through the CUTLASS kernel of the
  installed vLLM; where that is unavailable (no vLLM, a CPU tensor, shapes
  that are not multiples of 128) it expands the block scales and runs a bf16
  matmul.  `set_fp8_matmul("dequant")` forces the second path.  Compressed
  and uncompressed models share the layer, so decoded weights give identical
  logits.
* `fp8_model_from_config`: a transformers model from its config with every
  Linear of the decoder layers replaced by an `Fp8Linear` (random weights
  N(0, std) quantized per 128x128 tile, absmax -> 448, seeded per layer), or
  uninitialised for loading.
* `load_fp8_checkpoint`: the same from a local FP8 checkpoint directory
  (config.json + *.safetensors), read directly.
"""

import glob
import json
import os

import torch
import torch.nn as nn
import torch.nn.functional as F

E4M3_MAX = 448.0
BLOCK = 128

_MATMUL = {"mode": "auto", "ops": None, "quant": None, "failed": None}


def set_fp8_matmul(mode):
    """"auto" (block-scaled FP8 GEMM where available) or "dequant" (e4m3 ->
    bf16 expansion by the block scales, then a bf16 matmul)."""
    if mode not in ("auto", "dequant"):
        raise ValueError(mode)
    _MATMUL["mode"] = mode


def fp8_matmul_backend():
    """The FP8 GEMM that Fp8Linear uses on CUDA tensors: "cutlass-blockwise"
    or "dequant-bf16"."""
    return "cutlass-blockwise" if _cutlass_ops() is not None else "dequant-bf16"


def _cutlass_ops():
    if _MATMUL["mode"] != "auto" or _MATMUL["failed"]:
        return None
    if _MATMUL["ops"] is None:
        try:
            import vllm._custom_ops as ops
            from vllm.model_executor.layers.quantization.utils.fp8_utils import per_token_group_quant_fp8
            if not torch.cuda.is_available() or not ops.cutlass_scaled_mm_supports_block_fp8(
                    torch.cuda.get_device_capability()[0] * 10 + torch.cuda.get_device_capability()[1]):
                raise RuntimeError("no block-scaled FP8 GEMM for this device")
            _MATMUL["ops"], _MATMUL["quant"] = ops, per_token_group_quant_fp8
        except Exception as e:  # the bf16 expansion path serves both arms alike
            _MATMUL["failed"] = repr(e)
            return None
    return _MATMUL["ops"]


class Fp8Linear(nn.Module):
    def __init__(self, in_features, out_features, bias=False, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=torch.float8_e4m3fn,
                                               device=device), requires_grad=False)
        sr, sc = -(-out_features // BLOCK), -(-in_features // BLOCK)
        self.register_buffer("weight_scale_inv", torch.ones(sr, sc, dtype=torch.float32, device=device))
        self.bias = nn.Parameter(torch.zeros(out_features, device=device), requires_grad=False) if bias else None

    def dequantized(self, dtype=torch.bfloat16):
        o, i = self.out_features, self.in_features
        if o % BLOCK == 0 and i % BLOCK == 0:  # one broadcast multiply per 128x128 tile
            w = self.weight.view(o // BLOCK, BLOCK, i // BLOCK, BLOCK).to(dtype)
            return (w * self.weight_scale_inv.to(dtype)[:, None, :, None]).view(o, i)
        s = self.weight_scale_inv.repeat_interleave(BLOCK, 0)[:o].repeat_interleave(BLOCK, 1)[:, :i]
        return (self.weight.float() * s).to(dtype)

    def forward(self, x):
        o, i = self.out_features, self.in_features
        ops = _cutlass_ops() if x.is_cuda and o % BLOCK == 0 and i % BLOCK == 0 else None
        if ops is None:
            return F.linear(x, self.dequantized(x.dtype), self.bias)
        x2 = x.reshape(-1, i)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        xq, xs = _MATMUL["quant"](x2, BLOCK, column_major_scales=True, use_ue8m0=False)
        y = ops.cutlass_scaled_mm(xq, self.weight.t(), scale_a=xs, scale_b=self.weight_scale_inv.t(),
                                  out_dtype=x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y.reshape(*x.shape[:-1], o).to(x.dtype)

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, e4m3 128x128"


def quantize_block128(w):
    """fp32 [out, in] -> (e4m3 weight, f32 scale_inv per 128x128 tile), absmax -> 448."""
    o, i = w.shape
    ro, ri = -(-o // BLOCK) * BLOCK, -(-i // BLOCK) * BLOCK
    p = torch.zeros(ro, ri, dtype=torch.float32, device=w.device)
    p[:o, :i] = w
    tiles = p.view(ro // BLOCK, BLOCK, ri // BLOCK, BLOCK)
    amax = tiles.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = E4M3_MAX / amax
    q = (tiles * scale[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(ro, ri)[:o, :i].contiguous(), (1.0 / scale).float()


def _decoder_layers(model):
    inner = getattr(model, "model", model)
    return inner.layers


def replace_linears_with_fp8(model, device=None):
    """Swaps every nn.Linear inside the decoder layers for an Fp8Linear of the
    same shape (uninitialised).  Returns the swapped names."""
    names = []
    layers = _decoder_layers(model)
    for li, layer in enumerate(layers):
        for name, mod in list(layer.named_modules()):
            if isinstance(mod, nn.Linear):
                parent = layer
                parts = name.split(".")
                for p in parts[:-1]:
                    parent = getattr(parent, p)
                dev = device if device is not None else mod.weight.device
                setattr(parent, parts[-1], Fp8Linear(mod.in_features, mod.out_features, mod.bias is not None, dev))
                names.append(f"layers.{li}.{name}")
    return names


def fp8_model_from_config(config, device="cuda", seed=None, std=0.02, dtype=torch.bfloat16):
    """A causal LM from `config` with e4m3 Linear layers in every decoder
    layer.  seed=None leaves weights uninitialised (for loading); otherwise
    every weight is N(0, std) drawn from generator seed + k (k counts the
    model's parameters in order) and Linear weights are quantized per tile."""
    from transformers import AutoModelForCausalLM
    with torch.device(device):
        model = AutoModelForCausalLM.from_config(config, dtype=dtype)
    replace_linears_with_fp8(model, device)
    model.eval()
    if seed is not None:
        with torch.no_grad():
            k = 0
            for name, mod in model.named_modules():
                if isinstance(mod, Fp8Linear):
                    g = torch.Generator(device=device).manual_seed(seed + k)
                    w = torch.randn(mod.out_features, mod.in_features, generator=g, device=device) * std
                    q, s = quantize_block128(w)
                    mod.weight.data.copy_(q)
                    mod.weight_scale_inv.copy_(s)
                    k += 1
            for name, p in model.named_parameters(recurse=True):
                if p.dtype == torch.float8_e4m3fn:
                    continue
                g = torch.Generator(device=device).manual_seed(seed + k)
                k += 1
                if name.endswith("norm.weight") or p.ndim == 1:
                    p.fill_(1.0)
                else:
                    p.copy_((torch.randn(p.shape, generator=g, device=device) * std).to(p.dtype))
    return model


def load_fp8_checkpoint(path, device="cpu", dtype=torch.bfloat16):
    """Model of a local FP8 checkpoint directory (config.json with an fp8
    quantization_config, weights in *.safetensors), read without accelerate."""
    from safetensors.torch import load_file
    from transformers import AutoConfig
    config = AutoConfig.from_pretrained(path)
    model = fp8_model_from_config(config, device=device, seed=None, dtype=dtype)
    state = model.state_dict()
    for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
        for k, v in load_file(f, device=str(device)).items():
            if k in state and state[k].shape == v.shape:
                state[k].copy_(v.to(state[k].dtype))
    if getattr(config, "tie_word_embeddings", False):
        model.tie_weights()
    return model


def save_fp8_checkpoint(model, path):
    """Writes `model` as an FP8 checkpoint directory that load_fp8_checkpoint
    (and the compressor) read: config.json with an fp8 quantization_config
    and model.safetensors."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    cfg = model.config.to_dict()
    cfg["quantization_config"] = {"quant_method": "fp8", "activation_scheme": "dynamic",
                                  "weight_block_size": [BLOCK, BLOCK], "fmt": "e4m3"}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    tensors = {k: v.detach().contiguous().cpu() for k, v in model.state_dict().items()}
    if getattr(model.config, "tie_word_embeddings", False):
        tensors.pop("lm_head.weight", None)
    save_file(tensors, os.path.join(path, "model.safetensors"))
