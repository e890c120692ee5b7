"""Expert-parallel generation for the Qwen3-235B-A22B-shaped MoE set (config
5's generation run; the reference has only accelerate layer placement,
run.py:551-557).

One process per GPU.  Every rank holds a replica of each layer's attention
(and its own batch of prompts: data-parallel attention) and the experts it
owns, [r E/N, (r+1) E/N) of every layer.  An MoE layer routes each token to
its top-k experts, sends the token to the experts' owners with one NCCL
all-to-all, runs its local experts on what it received and sends the results
back with a second all-to-all; the owner-side outputs are combined with the
router weights in the tokens' original order.  No collective touches the
decode: a compressed rank decodes only its own streams.

Module paths follow the reference's `qwen3moe` pattern (dfloat/const.py):
`model.layers.N.self_attn` (q/k/v/o, 71,303,168 e4m3 weights) and
`model.layers.N.mlp.experts.M` (gate/up/down, 18,874,368), M the global
expert index.  Linear weights are e4m3 with 128x128 block scales
(ecf8_b200.fp8_model.Fp8Linear); router, norms, embeddings and lm_head bf16.
"""

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .fp8_model import Fp8Linear, quantize_block128


@dataclass
class MoEConfig:
    vocab_size: int = 151936
    hidden_size: int = 4096
    num_hidden_layers: int = 94
    num_attention_heads: int = 64
    num_key_value_heads: int = 4
    head_dim: int = 128
    num_experts: int = 128
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 1536
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6


class RMSNorm(nn.Module):
    def __init__(self, dim, eps, device):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=torch.bfloat16, device=device), requires_grad=False)

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight


def rotary(x, pos, theta):
    """x [B, H, T, D] rotated by positions pos [T] (half-split rotary)."""
    d = x.shape[-1]
    inv = 1.0 / theta ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d)
    ang = pos.float()[:, None] * inv[None]
    cos, sin = torch.cos(ang), torch.sin(ang)
    xf = x.float()
    a, b = xf[..., : d // 2], xf[..., d // 2:]
    return torch.cat((a * cos - b * sin, a * sin + b * cos), -1).to(x.dtype)


class Attention(nn.Module):
    def __init__(self, cfg, device):
        super().__init__()
        h, d = cfg.hidden_size, cfg.head_dim
        self.cfg = cfg
        self.q_proj = Fp8Linear(h, cfg.num_attention_heads * d, device=device)
        self.k_proj = Fp8Linear(h, cfg.num_key_value_heads * d, device=device)
        self.v_proj = Fp8Linear(h, cfg.num_key_value_heads * d, device=device)
        self.o_proj = Fp8Linear(cfg.num_attention_heads * d, h, device=device)
        self.q_norm = RMSNorm(d, cfg.rms_norm_eps, device)
        self.k_norm = RMSNorm(d, cfg.rms_norm_eps, device)

    def forward(self, x, cache, start):
        c = self.cfg
        b, t, _ = x.shape
        q = self.q_norm(self.q_proj(x).view(b, t, c.num_attention_heads, c.head_dim)).transpose(1, 2)
        k = self.k_norm(self.k_proj(x).view(b, t, c.num_key_value_heads, c.head_dim)).transpose(1, 2)
        v = self.v_proj(x).view(b, t, c.num_key_value_heads, c.head_dim).transpose(1, 2)
        pos = torch.arange(start, start + t, device=x.device)
        q, k = rotary(q, pos, c.rope_theta), rotary(k, pos, c.rope_theta)
        kc, vc = cache
        kc[:, :, start:start + t] = k
        vc[:, :, start:start + t] = v
        keys, vals = kc[:, :, : start + t], vc[:, :, : start + t]
        o = F.scaled_dot_product_attention(q, keys, vals, is_causal=t > 1, enable_gqa=True)
        return self.o_proj(o.transpose(1, 2).reshape(b, t, -1))


class Expert(nn.Module):
    def __init__(self, cfg, device):
        super().__init__()
        h, f = cfg.hidden_size, cfg.moe_intermediate_size
        self.gate_proj = Fp8Linear(h, f, device=device)
        self.up_proj = Fp8Linear(h, f, device=device)
        self.down_proj = Fp8Linear(f, h, device=device)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


def _all_to_all(send, send_counts, recv_counts, group):
    import torch.distributed as dist
    out = send.new_empty((int(sum(recv_counts)),) + tuple(send.shape[1:]))
    dist.all_to_all_single(out, send.contiguous(), list(recv_counts), list(send_counts), group=group)
    return out


class SparseMoE(nn.Module):
    """Top-k routed experts, sharded over ranks; `experts` holds this rank's
    (keys: global expert index).  `expert_loader`, when set (compressed
    model), is called with the global indices of the local experts that
    received tokens before they run."""

    def __init__(self, cfg, rank, world, device, group=None):
        super().__init__()
        self.cfg, self.rank, self.world, self.group = cfg, rank, world, group
        self.per = cfg.num_experts // world
        self.gate = nn.Linear(cfg.hidden_size, cfg.num_experts, bias=False, device=device, dtype=torch.bfloat16)
        self.experts = nn.ModuleDict({str(e): Expert(cfg, device)
                                      for e in range(rank * self.per, (rank + 1) * self.per)})
        self.expert_loader = None

    def forward(self, x):
        b, t, h = x.shape
        k = self.cfg.num_experts_per_tok
        xs = x.reshape(-1, h)
        n = xs.shape[0]
        probs = F.softmax(self.gate(xs).float(), dim=-1)
        topw, tope = probs.topk(k, dim=-1)
        topw = topw / topw.sum(-1, keepdim=True)
        flat_e = tope.reshape(-1)
        flat_tok = torch.arange(n, device=x.device).repeat_interleave(k)
        dest = flat_e // self.per
        order = torch.argsort(dest, stable=True)  # assignments grouped by owner rank, in token order
        send_x, send_e = xs[flat_tok[order]], flat_e[order]
        send_counts = torch.bincount(dest, minlength=self.world)
        if self.world > 1:
            import torch.distributed as dist
            recv_counts_t = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts_t, send_counts, group=self.group)
            sc, rc = send_counts.tolist(), recv_counts_t.tolist()
            recv_x = _all_to_all(send_x, sc, rc, self.group)
            recv_e = _all_to_all(send_e, sc, rc, self.group)
        else:
            recv_x, recv_e = send_x, send_e
        # Received assignments grouped by local expert (stable: each expert's
        # rows stay in arrival order), so each expert runs on one contiguous
        # slice; one host read of the per-expert counts per layer.
        first = self.rank * self.per
        by_e = torch.argsort(recv_e, stable=True)
        counts = torch.bincount(recv_e - first, minlength=self.per).tolist()
        used = [first + i for i, c in enumerate(counts) if c]
        if self.expert_loader is not None:
            self.expert_loader(used)
        xs_e = recv_x[by_e]
        ys_e = torch.empty_like(xs_e)
        off = 0
        for i, c in enumerate(counts):
            if c:
                ys_e[off:off + c] = self.experts[str(first + i)](xs_e[off:off + c])
                off += c
        out = torch.empty_like(recv_x)
        out[by_e] = ys_e
        back = _all_to_all(out, rc, sc, self.group) if self.world > 1 else out
        per_assign = torch.empty_like(back)
        per_assign[order] = back
        y = (per_assign.view(n, k, h).float() * topw.view(n, k, 1)).sum(1)  # fixed order: deterministic
        return y.to(x.dtype).view(b, t, h)


class DecoderLayer(nn.Module):
    def __init__(self, cfg, rank, world, device, group=None):
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device)
        self.self_attn = Attention(cfg, device)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device)
        self.mlp = SparseMoE(cfg, rank, world, device, group)

    def forward(self, x, cache, start):
        x = x + self.self_attn(self.input_layernorm(x), cache, start)
        return x + self.mlp(self.post_attention_layernorm(x))


class MoEBackbone(nn.Module):
    def __init__(self, cfg, rank, world, device, group=None):
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size, device=device, dtype=torch.bfloat16)
        self.layers = nn.ModuleList([DecoderLayer(cfg, rank, world, device, group)
                                     for _ in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device)


class Qwen3MoeEP(nn.Module):
    """Causal LM with expert-parallel MoE layers (this rank's shard)."""

    def __init__(self, cfg, rank=0, world=1, device="cuda", group=None):
        super().__init__()
        self.cfg = cfg
        self.model = MoEBackbone(cfg, rank, world, device, group)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False, device=device, dtype=torch.bfloat16)

    def new_cache(self, batch, max_len):
        c = self.cfg
        dev = self.lm_head.weight.device
        return [(torch.empty(batch, c.num_key_value_heads, max_len, c.head_dim, dtype=torch.bfloat16, device=dev),
                 torch.empty(batch, c.num_key_value_heads, max_len, c.head_dim, dtype=torch.bfloat16, device=dev))
                for _ in range(c.num_hidden_layers)]

    def forward(self, ids, caches, start):
        x = self.model.embed_tokens(ids)
        for layer, cache in zip(self.model.layers, caches):
            x = layer(x, cache, start)
        return self.lm_head(self.model.norm(x[:, -1:])).float()


def init_random(model, seed, std=0.02):
    """Seeded N(0, std) weights, identical on every rank for replicated
    modules: each module's generator seed comes from its name (experts by
    their global index), e4m3 128x128 block-quantized for Fp8Linear."""
    import zlib
    with torch.no_grad():
        for name, mod in model.named_modules():
            g = torch.Generator(device=mod.weight.device if hasattr(mod, "weight") else "cpu")
            g.manual_seed(seed * 1000003 + zlib.crc32(name.encode()))
            if isinstance(mod, Fp8Linear):
                w = torch.randn(mod.out_features, mod.in_features, generator=g, device=mod.weight.device) * std
                q, s = quantize_block128(w)
                mod.weight.data.copy_(q)
                mod.weight_scale_inv.copy_(s)
            elif isinstance(mod, (nn.Linear, nn.Embedding)):
                mod.weight.copy_((torch.randn(mod.weight.shape, generator=g, device=mod.weight.device) * std)
                                 .to(mod.weight.dtype))
    return model


def greedy_generate(model, ids, new_tokens, logit_sums=None):
    """Greedy decode of `new_tokens` tokens after the prompt `ids` [B, L];
    returns the new tokens [B, new_tokens].  Per-step float64 logit sums are
    appended to `logit_sums` when given."""
    b, l = ids.shape
    caches = model.new_cache(b, l + new_tokens)
    out = []
    with torch.no_grad():
        logits = model(ids, caches, 0)
        for step in range(new_tokens):
            if logit_sums is not None:
                logit_sums.append(logits.double().sum(dim=(1, 2)))
            nxt = logits[:, -1].argmax(-1, keepdim=True)
            out.append(nxt)
            if step + 1 < new_tokens:
                logits = model(nxt, caches, l + step)
    return torch.cat(out, 1)


_EXPERT_PARTS = ("down_proj", "gate_proj", "up_proj")  # sorted names: the stream's order


class ExpertStreamLoader:
    """The compressed experts of one MoE layer on this rank: each expert's
    gate/up/down weights are one ECF8 stream (with its prepared decode
    table).  Every owned expert has a fixed slot in `scratch` (slot i for the
    rank's i-th expert; all layers share the slots, as they run one after
    another), so its Linear weights point at the slot once, here, and its
    launch descriptor is checked and built once.  A call decodes the given
    experts into their slots with one batched launch on the current stream."""

    def __init__(self, moe, streams, scratch):
        from .run import _check_stream, _stream_struct
        self.moe = moe
        self.streams = streams  # global expert index -> stream dict (kept alive for the descriptors)
        self.scratch = scratch
        first = moe.rank * moe.per
        self.per = next(iter(streams.values()))["packed_other_4bits"].numel() * 2
        self.desc = {}
        for e, st in streams.items():
            flat = scratch[(e - first) * self.per:(e - first + 1) * self.per]
            table = st.get("decode_table")
            _check_stream(st, flat, scratch.device, table)
            self.desc[e] = _stream_struct(st, flat, table)
            expert = moe.experts[str(e)]
            off = 0
            for part in _EXPERT_PARTS:
                lin = getattr(expert, part)
                n = lin.out_features * lin.in_features
                lin.weight = flat[off:off + n].view(lin.out_features, lin.in_features)
                off += n

    def __call__(self, used):
        from . import _lib
        if not used:
            return
        arr = (_lib.Ecf8Stream * len(used))(*[self.desc[e] for e in used])
        cs = torch.cuda.current_stream(self.scratch.device)
        st = _lib.lib().ecf8_decode_batch_flags(arr, len(used), _lib.THREADS_PER_BLOCK, _lib.BYTES_PER_THREAD, 0,
                                                cs.cuda_stream)
        _lib.check(st, "ecf8_decode_batch_flags")


def _flat_fp8(modules):
    return torch.cat([m.weight.data.reshape(-1).view(torch.uint8) for m in modules]).view(torch.float8_e4m3fn)


def compress_ep_model(model, threads_per_block=512, bytes_per_thread=8):
    """Replaces this rank's FP8 weights by ECF8 streams: attention blocks get
    the decode-before-forward hook (one stream per `self_attn`), each MoE
    layer an ExpertStreamLoader (one stream per owned expert, decoded only
    when it receives tokens).  Returns the number of stream bytes."""
    from .codec import compress_fp8
    from .run import _process_compressed_tensor, build_decode_table
    total = 0
    scratch = None
    for li, layer in enumerate(model.model.layers):
        attn = layer.self_attn
        names = ["k_proj", "o_proj", "q_proj", "v_proj"]
        c = compress_fp8(_flat_fp8([getattr(attn, n) for n in names]))
        sizes = [getattr(attn, n).weight.numel() for n in names]
        split = torch.cumsum(torch.tensor(sizes, dtype=torch.int64), 0)[:-1]
        tensors = {"luts": c["luts"], "encoded": c["encoded"], "packed_other_4bits": c["packed_other_4bits"],
                   "output_positions": c["output_positions"].view(torch.uint8), "gaps": c["gaps"],
                   "split_positions": split}
        block = f"model.layers.{li}.self_attn"
        for key in ("luts", "packed_other_4bits", "output_positions", "gaps", "split_positions", "encoded"):
            _process_compressed_tensor(attn, key, tensors[key], f"{block}.{key}",
                                       {r"model\.layers\.\d+\.self_attn": names}, threads_per_block,
                                       bytes_per_thread)
        total += sum(tensors[k].numel() for k in ("luts", "encoded", "packed_other_4bits", "output_positions",
                                                 "gaps"))
        streams = {}
        for key, expert in layer.mlp.experts.items():
            parts = [getattr(expert, p) for p in _EXPERT_PARTS]
            s = compress_fp8(_flat_fp8(parts))
            s["decode_table"] = build_decode_table(s["luts"])
            for p in parts:
                del p.weight
            streams[int(key)] = s
            total += sum(s[k].numel() * s[k].element_size()
                         for k in ("luts", "encoded", "packed_other_4bits", "output_positions", "gaps"))
        per = next(iter(streams.values()))["packed_other_4bits"].numel() * 2
        if scratch is None or scratch.numel() < len(streams) * per:
            scratch = torch.empty(len(streams) * per, dtype=torch.float8_e4m3fn,
                                  device=next(iter(streams.values()))["encoded"].device)
        layer.mlp.expert_loader = ExpertStreamLoader(layer.mlp, streams, scratch)
    return total
