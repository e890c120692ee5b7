"""A FLUX.1-dev-shaped DiT with DiffSynth's module names (config 4).

The reference benchmarks ECF8 on DiffSynth's FLUX pipeline
(scripts/inference_dfsyn.py, dfloat/run/run.py:569-729), which is not
installed here.  This module rebuilds the DiT with the same block structure
and sub-module names, so the reference's FLUX pattern dict
(`diffsynth-flux-fp8`, dfloat/const.py:22-46) selects the same streams:

  dit.blocks.N          19 double-stream blocks: attn.{a,b}_to_qkv (3072 ->
                        9216), attn.{a,b}_to_out, ff_{a,b}.0 (3072 -> 12288),
                        ff_{a,b}.2 -> 226,492,416 e4m3 weights per stream
  dit.single_blocks.N   38 single-stream blocks: norm.linear (3072 -> 9216),
                        to_qkv_mlp (3072 -> 21504), proj_out (15360 -> 3072)
                        -> 141,557,760 e4m3 weights per stream

Those sub-Linears hold e4m3 weights with one per-tensor scale (absmax ->
448); the AdaLN modulation of the double blocks, the embedders and the final
layer stay bf16.  Attention is joint over [text, image] tokens with per-head
RMS-normalised q / k and 3-axis rotary position embedding (FLUX's 16/56/56
split of head_dim 128); activations are bf16.
"""

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

E4M3_MAX = 448.0


class Fp8TensorLinear(nn.Module):
    """e4m3 weight [out, in] with one f32 scale; forward casts the weight to
    the activation dtype times the scale (what DiffSynth's FP8 linear does on
    compute) and runs a bf16 matmul."""

    def __init__(self, in_features, out_features, bias=True, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=torch.float8_e4m3fn,
                                               device=device), requires_grad=False)
        self.register_buffer("weight_scale", torch.ones((), dtype=torch.float32, device=device))
        self.bias = nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16, device=device),
                                 requires_grad=False) if bias else None

    def forward(self, x):
        w = self.weight.to(x.dtype) * self.weight_scale.to(x.dtype)
        return F.linear(x, w, self.bias)


def _lin(i, o, fp8, device, bias=True):
    if fp8:
        return Fp8TensorLinear(i, o, bias, device)
    return nn.Linear(i, o, bias=bias, device=device, dtype=torch.bfloat16)


def _ln(x):
    return F.layer_norm(x, x.shape[-1:], eps=1e-6)


class RMSNorm(nn.Module):
    def __init__(self, dim, device):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, dtype=torch.bfloat16, device=device), requires_grad=False)

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * self.weight


def rope_freqs(ids, axes=(16, 56, 56), theta=10000.0):
    """cos / sin [N, head_dim/2] of FLUX's 3-axis rotary embedding for
    position ids [N, 3]."""
    parts = []
    for k, d in enumerate(axes):
        inv = 1.0 / theta ** (torch.arange(0, d, 2, device=ids.device, dtype=torch.float64) / d)
        parts.append(ids[:, k:k + 1].double() * inv[None])
    ang = torch.cat(parts, dim=-1)
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope(x, cos, sin):
    """x [B, H, N, D] rotated pairwise (x[2j], x[2j+1])."""
    xf = x.float().unflatten(-1, (-1, 2))
    a, b = xf[..., 0], xf[..., 1]
    out = torch.stack((a * cos - b * sin, a * sin + b * cos), dim=-1).flatten(-2)
    return out.to(x.dtype)


def joint_attention(q, k, v, cos, sin):
    """q, k, v [B, N, H, D] -> [B, N, H*D]."""
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
    o = F.scaled_dot_product_attention(q, k, v)
    return o.transpose(1, 2).flatten(2)


class AdaLayerNorm(nn.Module):
    def __init__(self, dim, n, fp8, device):
        super().__init__()
        self.linear = _lin(dim, n * dim, fp8, device)

    def forward(self, c):
        return self.linear(F.silu(c))


class DoubleAttention(nn.Module):
    def __init__(self, dim, heads, device):
        super().__init__()
        self.heads = heads
        self.a_to_qkv = _lin(dim, 3 * dim, True, device)
        self.b_to_qkv = _lin(dim, 3 * dim, True, device)
        self.a_to_out = _lin(dim, dim, True, device)
        self.b_to_out = _lin(dim, dim, True, device)
        hd = dim // heads
        self.norm_q_a, self.norm_k_a = RMSNorm(hd, device), RMSNorm(hd, device)
        self.norm_q_b, self.norm_k_b = RMSNorm(hd, device), RMSNorm(hd, device)

    def forward(self, img, txt, cos, sin):
        qa, ka, va = self.a_to_qkv(img).unflatten(-1, (3, self.heads, -1)).unbind(2)
        qb, kb, vb = self.b_to_qkv(txt).unflatten(-1, (3, self.heads, -1)).unbind(2)
        q = torch.cat((self.norm_q_b(qb), self.norm_q_a(qa)), 1)
        k = torch.cat((self.norm_k_b(kb), self.norm_k_a(ka)), 1)
        v = torch.cat((vb, va), 1)
        o = joint_attention(q, k, v, cos, sin)
        nt = txt.shape[1]
        return self.a_to_out(o[:, nt:]), self.b_to_out(o[:, :nt])


class DoubleBlock(nn.Module):
    def __init__(self, dim, heads, device):
        super().__init__()
        self.norm1_a = AdaLayerNorm(dim, 6, False, device)
        self.norm1_b = AdaLayerNorm(dim, 6, False, device)
        self.attn = DoubleAttention(dim, heads, device)
        self.ff_a = nn.Sequential(_lin(dim, 4 * dim, True, device), nn.GELU(approximate="tanh"),
                                  _lin(4 * dim, dim, True, device))
        self.ff_b = nn.Sequential(_lin(dim, 4 * dim, True, device), nn.GELU(approximate="tanh"),
                                  _lin(4 * dim, dim, True, device))

    def forward(self, img, txt, c, cos, sin):
        sa, ca, ga, sma, cma, gma = self.norm1_a(c)[:, None].chunk(6, dim=-1)
        sb, cb, gb, smb, cmb, gmb = self.norm1_b(c)[:, None].chunk(6, dim=-1)
        ia, ta = self.attn(_ln(img) * (1 + ca) + sa, _ln(txt) * (1 + cb) + sb, cos, sin)
        img = img + ga * ia
        txt = txt + gb * ta
        img = img + gma * self.ff_a(_ln(img) * (1 + cma) + sma)
        txt = txt + gmb * self.ff_b(_ln(txt) * (1 + cmb) + smb)
        return img, txt


class SingleAdaNorm(nn.Module):
    def __init__(self, dim, device):
        super().__init__()
        self.linear = _lin(dim, 3 * dim, True, device)

    def forward(self, c):
        return self.linear(F.silu(c))


class SingleBlock(nn.Module):
    def __init__(self, dim, heads, device):
        super().__init__()
        self.heads, self.dim = heads, dim
        self.norm = SingleAdaNorm(dim, device)
        self.to_qkv_mlp = _lin(dim, 3 * dim + 4 * dim, True, device)
        self.proj_out = _lin(dim + 4 * dim, dim, True, device)
        hd = dim // heads
        self.norm_q_a, self.norm_k_a = RMSNorm(hd, device), RMSNorm(hd, device)

    def forward(self, x, c, cos, sin):
        shift, scale, gate = self.norm(c)[:, None].chunk(3, dim=-1)
        h = self.to_qkv_mlp(_ln(x) * (1 + scale) + shift)
        qkv, mlp = h[..., : 3 * self.dim], h[..., 3 * self.dim:]
        q, k, v = qkv.unflatten(-1, (3, self.heads, -1)).unbind(2)
        o = joint_attention(self.norm_q_a(q), self.norm_k_a(k), v, cos, sin)
        return x + gate * self.proj_out(torch.cat((o, F.gelu(mlp, approximate="tanh")), -1))


def timestep_embedding(t, dim=256, max_period=10000.0):
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t.float()[:, None] * 1000.0 * freqs[None]
    return torch.cat((torch.cos(args), torch.sin(args)), -1)


class MLPEmbedder(nn.Module):
    def __init__(self, i, dim, device):
        super().__init__()
        self.l1 = nn.Linear(i, dim, device=device, dtype=torch.bfloat16)
        self.l2 = nn.Linear(dim, dim, device=device, dtype=torch.bfloat16)

    def forward(self, x):
        return self.l2(F.silu(self.l1(x)))


class FluxDiT(nn.Module):
    def __init__(self, dim=3072, heads=24, n_double=19, n_single=38, in_channels=64, text_dim=4096,
                 pooled_dim=768, device=None):
        super().__init__()
        self.x_embedder = nn.Linear(in_channels, dim, device=device, dtype=torch.bfloat16)
        self.context_embedder = nn.Linear(text_dim, dim, device=device, dtype=torch.bfloat16)
        self.time_embedder = MLPEmbedder(256, dim, device)
        self.guidance_embedder = MLPEmbedder(256, dim, device)
        self.pooled_text_embedder = MLPEmbedder(pooled_dim, dim, device)
        self.blocks = nn.ModuleList([DoubleBlock(dim, heads, device) for _ in range(n_double)])
        self.single_blocks = nn.ModuleList([SingleBlock(dim, heads, device) for _ in range(n_single)])
        self.final_norm = nn.Linear(dim, 2 * dim, device=device, dtype=torch.bfloat16)
        self.final_proj_out = nn.Linear(dim, in_channels, device=device, dtype=torch.bfloat16)

    def forward(self, latents, text, pooled, t, guidance, cos, sin):
        c = (self.time_embedder(timestep_embedding(t).to(torch.bfloat16))
             + self.guidance_embedder(timestep_embedding(guidance).to(torch.bfloat16))
             + self.pooled_text_embedder(pooled))
        img, txt = self.x_embedder(latents), self.context_embedder(text)
        for blk in self.blocks:
            img, txt = blk(img, txt, c, cos, sin)
        x = torch.cat((txt, img), 1)
        for blk in self.single_blocks:
            x = blk(x, c, cos, sin)
        img = x[:, txt.shape[1]:]
        shift, scale = self.final_norm(F.silu(c))[:, None].chunk(2, dim=-1)
        return self.final_proj_out(_ln(img) * (1 + scale) + shift)


class FluxDiTPipeline(nn.Module):
    """Holds the DiT as `dit`, so that block names are `dit.blocks.N` /
    `dit.single_blocks.N` as in DiffSynth's FluxImagePipeline."""

    def __init__(self, dit):
        super().__init__()
        self.dit = dit


def quantize_per_tensor(w):
    amax = w.abs().max().clamp_min(1e-12)
    scale = E4M3_MAX / amax
    return (w * scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn), (1.0 / scale).float()


def flux_dit_pipeline(device="cuda", seed=0, std=0.02, **shape):
    """A FluxDiTPipeline with random weights: every weight N(0, std) from
    generator seed + k (k counts modules in order), e4m3 per-tensor for the
    compressed sub-Linears, bf16 elsewhere; norms 1, biases 0."""
    with torch.device(device):
        pipe = FluxDiTPipeline(FluxDiT(device=device, **shape))
    pipe.eval()
    with torch.no_grad():
        for k, (name, mod) in enumerate(pipe.named_modules()):
            g = torch.Generator(device=device).manual_seed(seed + k)
            if isinstance(mod, Fp8TensorLinear):
                w = torch.randn(mod.out_features, mod.in_features, generator=g, device=device) * std
                q, s = quantize_per_tensor(w)
                mod.weight.data.copy_(q)
                mod.weight_scale.copy_(s)
                del w
                if mod.bias is not None:
                    mod.bias.zero_()
            elif isinstance(mod, nn.Linear):
                mod.weight.copy_((torch.randn(mod.weight.shape, generator=g, device=device) * std).to(mod.weight.dtype))
                if mod.bias is not None:
                    mod.bias.zero_()
    return pipe


def position_ids(n_text, h, w, device):
    """FLUX's ids: text tokens (0, 0, 0), image token (0, row, col)."""
    txt = torch.zeros(n_text, 3, device=device)
    r = torch.arange(h, device=device).repeat_interleave(w)
    c = torch.arange(w, device=device).repeat(h)
    img = torch.stack((torch.zeros_like(r), r, c), 1).float()
    return torch.cat((txt, img), 0)
