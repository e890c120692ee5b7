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
* `Fp8FusedExperts`: the FP8 form of transformers' fused MoE experts
  (`Qwen3MoeExperts`, whose experts are 3-D `gate_up_proj` / `down_proj`
  parameters), e4m3 with 128x128 block scales per expert.  Its state dict
  uses the per-expert keys of FP8 checkpoints and of the reference's
  compressed layout (`...mlp.experts.M.{gate,up,down}_proj.weight[_scale_inv]`,
  and `...mlp.experts.M.{luts,encoded,...}` once compressed: one ECF8 stream
  per expert, dfloat/const.py:15-21).  Compressed, its forward decodes only
  the experts the router picked, in one batched launch.
* `fp8_model_from_config`: a transformers model from its config with every
  Linear of the decoder layers replaced by an `Fp8Linear` and every fused
  expert block by an `Fp8FusedExperts` (random weights N(0, std) quantized per
  128x128 tile, absmax -> 448, seeded per layer), or uninitialised for loading.
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


def dequantize_block128(weight, scale_inv, dtype=torch.bfloat16):
    """e4m3 [out, in] times its 128x128 tile scales, in `dtype`."""
    o, i = weight.shape
    if o % BLOCK == 0 and i % BLOCK == 0:  # one broadcast multiply per 128x128 tile
        w = weight.reshape(o // BLOCK, BLOCK, i // BLOCK, BLOCK).to(dtype)
        return (w * scale_inv.to(dtype)[:, None, :, None]).reshape(o, i)
    s = scale_inv.repeat_interleave(BLOCK, 0)[:o].repeat_interleave(BLOCK, 1)[:, :i]
    return (weight.float() * s).to(dtype)


def fp8_linear(x, weight, scale_inv, bias=None):
    """x @ (weight * tile scales)^T for an e4m3 weight [out, in] with 128x128
    block scales: the block-scaled FP8 GEMM (activations quantized per 1x128
    group) where available, else the bf16 expansion."""
    o, i = weight.shape
    ops = _cutlass_ops() if x.is_cuda and o % BLOCK == 0 and i % BLOCK == 0 else None
    if ops is None:
        return F.linear(x, dequantize_block128(weight, scale_inv, x.dtype), bias)
    x2 = x.reshape(-1, i)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    xq, xs = _MATMUL["quant"](x2, BLOCK, column_major_scales=True, use_ue8m0=False)
    y = ops.cutlass_scaled_mm(xq, weight.t(), scale_a=xs, scale_b=scale_inv.t(),
                              out_dtype=x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16)
    if bias is not None:
        y = y + bias.to(y.dtype)
    return y.reshape(*x.shape[:-1], o).to(x.dtype)


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
        return dequantize_block128(self.weight, self.weight_scale_inv, dtype)

    def forward(self, x):
        return fp8_linear(x, self.weight, self.weight_scale_inv, self.bias)

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, e4m3 128x128"


_STREAM_KEYS = ("luts", "encoded", "packed_other_4bits", "output_positions", "gaps", "split_positions")
_DENSE_KEYS = ("gate_proj.weight", "up_proj.weight", "down_proj.weight", "gate_proj.weight_scale_inv",
               "up_proj.weight_scale_inv", "down_proj.weight_scale_inv")


class _ExpertLinearView:
    """One expert's sub-Linear inside a fused parameter, as the compressor's
    block walk sees a Linear: a `weight` (a view) and its shape."""

    def __init__(self, weight):
        self.weight = weight
        self.out_features, self.in_features = weight.shape


class Fp8FusedExperts(nn.Module):
    """transformers' fused MoE experts (Qwen3MoeExperts: `gate_up_proj`
    [E, 2I, H], `down_proj` [E, H, I], gate rows before up rows) in e4m3 with
    128x128 block scales per expert.  Same forward contract and the same
    routing loop as transformers' eager implementation; each expert's matmuls
    go through `fp8_linear`.

    Compressed (`add_expert_stream`), expert M is one ECF8 stream: its
    down, gate and up weights concatenated in that (sorted-name) order, which
    is down_proj[M] followed by gate_up_proj[M].  The dense parameters are
    dropped once every expert has its stream; the forward then decodes the
    experts the router picked, in one batched launch, into the per-device
    scratch (the same TensorManager buffer the block hooks use: the block's
    attention has run by then) and uses views of it."""

    def __init__(self, num_experts, hidden_size, intermediate_size, act_fn, device=None):
        super().__init__()
        if hidden_size % BLOCK or intermediate_size % BLOCK:
            raise ValueError("expert sizes must be multiples of 128 for 128x128 block scales")
        self.num_experts, self.hidden_dim, self.intermediate_dim = num_experts, hidden_size, intermediate_size
        e, h, i = num_experts, hidden_size, intermediate_size
        self.gate_up_proj = nn.Parameter(torch.empty(e, 2 * i, h, dtype=torch.float8_e4m3fn, device=device),
                                         requires_grad=False)
        self.down_proj = nn.Parameter(torch.empty(e, h, i, dtype=torch.float8_e4m3fn, device=device),
                                      requires_grad=False)
        self.register_buffer("gate_up_proj_scale_inv",
                             torch.ones(e, 2 * i // BLOCK, h // BLOCK, dtype=torch.float32, device=device))
        self.register_buffer("down_proj_scale_inv",
                             torch.ones(e, h // BLOCK, i // BLOCK, dtype=torch.float32, device=device))
        self.act_fn = act_fn
        self.compressed = set()
        self.threads_per_block, self.bytes_per_thread = 512, 8

    # -- per-expert views -----------------------------------------------------
    def expert_layers(self, m, prefix):
        """{sub-Linear name: view} of expert m's dense weights, in sorted order."""
        i = self.intermediate_dim
        return {f"{prefix}.down_proj": _ExpertLinearView(self.down_proj.data[m]),
                f"{prefix}.gate_proj": _ExpertLinearView(self.gate_up_proj.data[m, :i]),
                f"{prefix}.up_proj": _ExpertLinearView(self.gate_up_proj.data[m, i:])}

    def _dense_view(self, m, key):
        i, k = self.intermediate_dim, self.intermediate_dim // BLOCK
        return {"gate_proj.weight": lambda: self.gate_up_proj.data[m, :i],
                "up_proj.weight": lambda: self.gate_up_proj.data[m, i:],
                "down_proj.weight": lambda: self.down_proj.data[m],
                "gate_proj.weight_scale_inv": lambda: self.gate_up_proj_scale_inv[m, :k],
                "up_proj.weight_scale_inv": lambda: self.gate_up_proj_scale_inv[m, k:],
                "down_proj.weight_scale_inv": lambda: self.down_proj_scale_inv[m]}[key]()

    def _has_dense(self):
        return isinstance(getattr(self, "gate_up_proj", None), torch.Tensor)

    def load_expert_tensor(self, m, key, value, threads_per_block=512, bytes_per_thread=8):
        """Takes one per-expert checkpoint tensor: a dense weight or scale
        (copied into the fused parameter) or a stream buffer."""
        if key in _STREAM_KEYS:
            self.add_expert_stream(m, key, value, threads_per_block, bytes_per_thread)
            return
        if key.endswith(".weight") and not self._has_dense():
            raise ValueError(f"expert {m}: dense {key} after the experts were compressed")
        dst = self._dense_view(m, key)
        if dst.shape != value.shape:
            raise ValueError(f"expert {m} {key}: shape {tuple(value.shape)}, expected {tuple(dst.shape)}")
        dst.copy_(value.to(dst.dtype))

    def add_expert_stream(self, m, key, value, threads_per_block=512, bytes_per_thread=8):
        """Registers one stream buffer of expert m; once every expert has its
        `encoded` buffer the dense parameters are dropped."""
        if not 0 <= m < self.num_experts:
            raise ValueError(f"expert {m} out of range")
        self.threads_per_block, self.bytes_per_thread = threads_per_block, bytes_per_thread
        if key == "split_positions":
            want = [self.hidden_dim * self.intermediate_dim, 2 * self.hidden_dim * self.intermediate_dim]
            got = [int(x) for x in (value.tolist() if isinstance(value, torch.Tensor) else value)]
            if got != want:
                raise ValueError(f"expert {m}: split positions {got}, expected {want} (down, gate, up)")
            return
        self.register_buffer(f"ecf8_{m}_{key}", value)
        if key == "encoded":
            self.compressed.add(m)
            if len(self.compressed) == self.num_experts and self._has_dense():
                del self.gate_up_proj
                del self.down_proj

    def _stream(self, m):
        s = {k: getattr(self, f"ecf8_{m}_{k}") for k in _STREAM_KEYS if k != "split_positions"}
        s["decode_table"] = getattr(self, f"ecf8_{m}_decode_table", None)
        return s

    # -- state dict in the per-expert checkpoint layout -------------------------
    def _save_to_state_dict(self, destination, prefix, keep_vars):
        for m in range(self.num_experts):
            if m in self.compressed:
                for k in _STREAM_KEYS:
                    if k == "split_positions":
                        hi = self.hidden_dim * self.intermediate_dim
                        destination[f"{prefix}{m}.{k}"] = torch.tensor([hi, 2 * hi], dtype=torch.int64)
                    else:
                        destination[f"{prefix}{m}.{k}"] = getattr(self, f"ecf8_{m}_{k}")
                keys = [k for k in _DENSE_KEYS if k.endswith("_scale_inv")]
            else:
                keys = _DENSE_KEYS
            for k in keys:
                t = self._dense_view(m, k)
                destination[f"{prefix}{m}.{k}"] = t if keep_vars else t.detach()

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        for name in list(state_dict):
            if not name.startswith(prefix):
                continue
            rest = name[len(prefix):]
            head, _, key = rest.partition(".")
            if head.isdigit() and (key in _STREAM_KEYS or key in _DENSE_KEYS):
                self.load_expert_tensor(int(head), key, state_dict[name])
            elif not rest.startswith("ecf8_"):
                unexpected_keys.append(name)

    # -- forward ----------------------------------------------------------------
    def expert_weights(self, experts):
        """[(gate_up [2I, H], down [H, I])] e4m3 for the given experts: views of
        the dense parameters, or of their decoded streams (the compressed ones
        among them in one batched launch)."""
        coded = [m for m in experts if m in self.compressed]
        views = {m: (self.gate_up_proj[m], self.down_proj[m]) for m in experts if m not in self.compressed}
        if coded:
            from .run import TensorManager, build_decode_table, decode_streams
            h, i = self.hidden_dim, self.intermediate_dim
            per = 3 * h * i
            pad = (per + 255) & ~255
            dev = getattr(self, f"ecf8_{coded[0]}_encoded").device
            fresh = False
            for m in coded:
                if getattr(self, f"ecf8_{m}_decode_table", None) is None:
                    self.register_buffer(f"ecf8_{m}_decode_table",
                                         build_decode_table(getattr(self, f"ecf8_{m}_luts")), persistent=False)
                    fresh = True
            scratch = TensorManager.get_tensor(dev, len(coded) * pad)
            outs = [scratch[j * pad:j * pad + per] for j in range(len(coded))]
            decode_streams([self._stream(m) for m in coded], [o.view(torch.uint8) for o in outs],
                           self.threads_per_block, self.bytes_per_thread, overlap_previous=not fresh)
            for m, o in zip(coded, outs):
                views[m] = (o[h * i:].view(2 * i, h), o[:h * i].view(h, i))
        return [views[m] for m in experts]

    def forward(self, hidden_states, top_k_index, top_k_weights):
        final = torch.zeros_like(hidden_states)
        with torch.no_grad():
            mask = F.one_hot(top_k_index, num_classes=self.num_experts).permute(2, 1, 0)
            hit = torch.greater(mask.sum(dim=(-1, -2)), 0).nonzero()[:, 0].tolist()
        for m, (gate_up, down) in zip(hit, self.expert_weights(hit)):
            top_k_pos, token_idx = torch.where(mask[m])
            gate, up = fp8_linear(hidden_states[token_idx], gate_up, self.gate_up_proj_scale_inv[m]).chunk(2, dim=-1)
            cur = fp8_linear(self.act_fn(gate) * up, down, self.down_proj_scale_inv[m])
            cur = cur * top_k_weights[token_idx, top_k_pos, None]
            final.index_add_(0, token_idx, cur.to(final.dtype))
        return final

    def extra_repr(self):
        return (f"num_experts={self.num_experts}, hidden={self.hidden_dim}, intermediate={self.intermediate_dim}, "
                f"e4m3 128x128, compressed={len(self.compressed)}")


def fused_experts_owner(model, name):
    """(Fp8FusedExperts module, expert index, key) when `name` addresses one
    expert's tensor inside a fused expert block ("...experts.M.key"), else None."""
    parts = name.split(".")
    mod = model
    for j, part in enumerate(parts):
        if isinstance(mod, Fp8FusedExperts):
            if part.isdigit() and j + 1 < len(parts):
                return mod, int(part), ".".join(parts[j + 1:])
            return None
        mod = getattr(mod, part, None)
        if mod is None or not isinstance(mod, nn.Module):
            return None
    return None


def replace_fused_experts_with_fp8(model, device=None):
    """Swaps every fused expert block (a module with 3-D `gate_up_proj` /
    `down_proj`, e.g. Qwen3MoeExperts) for an Fp8FusedExperts of the same
    shape (uninitialised).  Returns the swapped names."""
    names = []
    for name, mod in list(model.named_modules()):
        gu = getattr(mod, "gate_up_proj", None)
        if isinstance(mod, Fp8FusedExperts) or not isinstance(gu, torch.Tensor) or gu.dim() != 3:
            continue
        parent = model
        parts = name.split(".")
        for p in parts[:-1]:
            parent = getattr(parent, p)
        e, two_i, h = gu.shape
        dev = device if device is not None else gu.device
        setattr(parent, parts[-1], Fp8FusedExperts(e, h, two_i // 2, mod.act_fn, dev))
        names.append(name)
    return names


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
    replace_fused_experts_with_fp8(model, device)
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
                elif isinstance(mod, Fp8FusedExperts):
                    for m in range(mod.num_experts):
                        for key, (o, i) in (("gate_proj", (mod.intermediate_dim, mod.hidden_dim)),
                                            ("up_proj", (mod.intermediate_dim, mod.hidden_dim)),
                                            ("down_proj", (mod.hidden_dim, mod.intermediate_dim))):
                            g = torch.Generator(device=device).manual_seed(seed + k)
                            q, s = quantize_block128(torch.randn(o, i, generator=g, device=device) * std)
                            mod.load_expert_tensor(m, key + ".weight", q)
                            mod.load_expert_tensor(m, key + ".weight_scale_inv", s)
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
