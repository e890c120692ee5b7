"""End-to-end LLM generation with on-the-fly ECF8 decode, compressed vs
uncompressed (config 3; the reference's scripts/inference_llm.py).

    python -m ecf8_b200.inference_llm --synthetic --batch_size 16 --prompt_len 128 --num_tokens 1024

--synthetic builds the random-init Qwen3-8B architecture (vocab 151,936,
hidden 4096, 36 layers, 32 query / 8 KV heads of 128, SwiGLU 12,288, RoPE
theta 1e6) with e4m3 Linear weights (N(0, 0.02), 128x128 block scales);
otherwise --repo_id is a local FP8 checkpoint directory.  Prompts are
batch_size x prompt_len uniformly random token ids (seeded).

Both arms run in one process on one model: first the uncompressed FP8 model,
then the same model with its decoder layers compressed in place (each layer
decoded into the shared scratch by the forward-pre-hook, as
DFloatModel.from_pretrained sets it up).  Timing follows the reference
(inference_llm.py:109-160): a warm-up forward without cache, then
`generate` between two synchronisations, greedy instead of sampling so that
the arms are comparable; each arm first runs one untimed generation of the
same length, so that neither pays the allocator's first-growth cost.  Every step's logits are checked: the first steps in
full, all steps by a per-row float64 sum, plus the generated tokens.

Both arms use the same FP8 Linear (ecf8_b200.fp8_model.Fp8Linear: a
block-scaled FP8 GEMM reading e4m3 weights directly, or with
--fp8_matmul dequant the e4m3 -> bf16 expansion and a bf16 matmul), so
identical decoded weights must give identical logits.
"""

import argparse
import json
import time

import torch


def qwen3_8b_config(num_hidden_layers=36):
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                       num_hidden_layers=num_hidden_layers, num_attention_heads=32, num_key_value_heads=8,
                       head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6, max_position_embeddings=40960,
                       tie_word_embeddings=False, hidden_act="silu")


class LogitsRecorder:
    """A logits processor that keeps every step's logits on the GPU as a
    per-row float64 sum, and the first `keep` steps in full; it changes
    nothing, so greedy decoding is unaffected."""

    def __init__(self, keep=4):
        self.keep = keep
        self.sums = []
        self.full = []

    def __call__(self, input_ids, scores):
        self.sums.append(scores.double().sum(dim=-1))
        if len(self.full) < self.keep:
            self.full.append(scores.detach().clone())
        return scores


def _gen_config(n):
    from transformers import GenerationConfig
    return GenerationConfig(max_new_tokens=n, min_new_tokens=n, do_sample=False, eos_token_id=None,
                            pad_token_id=0, use_cache=True)


def generate_timed(model, input_ids, num_tokens, keep=4, warm_tokens=None):
    """One timed greedy generation of exactly `num_tokens` new tokens, after a
    warm-up forward without cache (inference_llm.py:109-114) and a warm-up
    generation of the same length (default): the first generation in a
    process grows the allocator's blocks for every KV-cache length, which cost
    the first of the two arms several times its steady-state step time."""
    warm_tokens = num_tokens if warm_tokens is None else warm_tokens
    from transformers import LogitsProcessorList
    rec = LogitsRecorder(keep)
    gen = _gen_config(num_tokens)
    mask = torch.ones_like(input_ids)
    with torch.no_grad():
        model(input_ids=input_ids, use_cache=False)
        if warm_tokens:
            model.generate(input_ids=input_ids, attention_mask=mask, generation_config=_gen_config(warm_tokens))
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.time()
    start.record()
    with torch.no_grad():
        out = model.generate(input_ids=input_ids, attention_mask=mask, generation_config=gen,
                             logits_processor=LogitsProcessorList([rec]))
    end.record()
    torch.cuda.synchronize()
    wall = time.time() - t0
    tokens = out[:, input_ids.shape[1]:]
    return {
        "latency_s": wall,
        "device_s": start.elapsed_time(end) / 1e3,
        "tokens_per_s": tokens.numel() / wall,
        "ms_per_step": wall / num_tokens * 1e3,
        "peak_hbm_mb": torch.cuda.max_memory_allocated() / 2**20,
        "allocated_mb": torch.cuda.memory_allocated() / 2**20,
        "new_tokens": tokens.shape[1],
    }, tokens, torch.stack(rec.sums), rec.full


def _model_bytes(model):
    fp8 = sum(p.numel() for p in model.parameters() if p.dtype == torch.float8_e4m3fn)
    streams = 0
    for m in model.modules():
        for key in ("luts", "encoded", "packed_other_4bits", "output_positions", "gaps"):
            b = m._buffers.get(key)
            if b is not None:
                streams += b.numel() * b.element_size()
    return fp8, streams


def main(argv=None):
    ap = argparse.ArgumentParser(description="Compressed vs uncompressed FP8 generation (config 3).")
    ap.add_argument("--repo_id", type=str, default=None, help="local FP8 checkpoint directory")
    ap.add_argument("--synthetic", action="store_true", help="random-init Qwen3-8B architecture")
    ap.add_argument("--num_layers", type=int, default=36, help="decoder layers of --synthetic")
    ap.add_argument("--batch_size", type=int, default=16)
    ap.add_argument("--prompt_len", type=int, default=128)
    ap.add_argument("--num_tokens", type=int, default=1024)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--no_compress", action="store_true", help="uncompressed arm only")
    ap.add_argument("--compressed_only", action="store_true", help="compressed arm only")
    ap.add_argument("--keep", type=int, default=4, help="steps whose full logits are compared")
    ap.add_argument("--warm_tokens", type=int, default=None, help="warm-up generation length (default: num_tokens)")
    ap.add_argument("--prefetch", action="store_true",
                    help="compressed arm: decode each layer one layer ahead on a side stream")
    ap.add_argument("--prefetch_ctas", type=int, default=0,
                    help="with --prefetch: CTAs of each side-stream decode (0: one per SM)")
    ap.add_argument("--fp8_matmul", choices=["auto", "dequant"], default="auto",
                    help="auto: block-scaled FP8 GEMM on e4m3 weights; dequant: bf16 expansion + bf16 matmul")
    args = ap.parse_args(argv)
    from .compress import compress_model_in_place
    from .fp8_model import fp8_matmul_backend, fp8_model_from_config, load_fp8_checkpoint, set_fp8_matmul
    set_fp8_matmul(args.fp8_matmul)
    from .run import TensorManager
    dev = torch.device("cuda", torch.cuda.current_device())
    t0 = time.time()
    if args.synthetic or args.repo_id is None:
        model = fp8_model_from_config(qwen3_8b_config(args.num_layers), device=dev, seed=args.seed)
        workload = f"config 3: random-init Qwen3-8B architecture ({args.num_layers} layers), FP8 linears"
    else:
        model = load_fp8_checkpoint(args.repo_id, device=dev)
        workload = f"FP8 checkpoint {args.repo_id}"
    model.eval()
    build_s = time.time() - t0
    g = torch.Generator(device=dev).manual_seed(args.seed)
    ids = torch.randint(0, model.config.vocab_size, (args.batch_size, args.prompt_len), generator=g, device=dev)
    fp8_bytes, _ = _model_bytes(model)
    line = {"workload": workload, "batch_size": args.batch_size, "prompt_len": args.prompt_len,
            "new_tokens": args.num_tokens, "decoding": "greedy", "model_build_s": round(build_s, 1),
            "fp8_matmul": fp8_matmul_backend()}
    ref = None
    if not args.compressed_only:
        res, tokens, sums, full = generate_timed(model, ids, args.num_tokens, args.keep, args.warm_tokens)
        line["uncompressed"] = {k: round(v, 3) if isinstance(v, float) else v for k, v in res.items()}
        ref = (tokens, sums, full)
    if not args.no_compress:
        t1 = time.time()
        compress_model_in_place(model)
        if args.prefetch:
            from .run import enable_decode_prefetch
            enable_decode_prefetch(model, ctas=args.prefetch_ctas)
        line["decode_prefetch"] = bool(args.prefetch)
        if args.prefetch:
            line["decode_prefetch_ctas"] = args.prefetch_ctas
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        TensorManager.clear_device()
        line["compress_s"] = round(time.time() - t1, 1)
        _, stream_bytes = _model_bytes(model)
        line["fp8_weight_bytes"] = fp8_bytes
        line["ecf8_stream_bytes"] = stream_bytes
        res, tokens, sums, full = generate_timed(model, ids, args.num_tokens, args.keep, args.warm_tokens)
        line["compressed"] = {k: round(v, 3) if isinstance(v, float) else v for k, v in res.items()}
        if ref is not None:
            line["identical_tokens"] = bool(torch.equal(tokens, ref[0]))
            line["identical_logit_sums_all_steps"] = bool(torch.equal(sums, ref[1]))
            line["identical_full_logits_first_steps"] = bool(all(torch.equal(a, b) for a, b in zip(full, ref[2])))
            line["compressed_vs_uncompressed_tokens_per_s"] = round(
                line["compressed"]["tokens_per_s"] / line["uncompressed"]["tokens_per_s"], 4)
    print(json.dumps(line), flush=True)
    return line


if __name__ == "__main__":
    main()
