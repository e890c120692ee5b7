"""Expert-parallel generation, compressed vs uncompressed (config 5's
generation run), one process per GPU:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m ecf8_b200.inference_moe --layers 94 --batch 16 --prompt_len 128 --new_tokens 32

Every rank builds the Qwen3-235B-A22B-shaped model's replicated parts and its
own experts (seeded random N(0, 0.02), e4m3 128x128 block scales; identical
replicas on all ranks), takes its own batch of random prompt ids and
generates greedily; MoE layers exchange tokens with NCCL all-to-all
(ecf8_b200.moe_ep).  The uncompressed arm runs first, then the same model
with every attention block and owned expert compressed in place.  Each arm
is warmed up, then timed between a barrier and a synchronisation on every
rank; the time is the maximum over ranks.  Tokens and every step's logits
(float64 sums) must be identical between the arms on every rank.
`--cpu` runs on gloo with CPU tensors (uncompressed arm only: the decode needs
a GPU) for testing the exchange.
"""

import argparse
import datetime
import json
import os
import time

import torch
import torch.distributed as dist


def _timed(model, ids, new_tokens, world, dev):
    from .moe_ep import greedy_generate
    greedy_generate(model, ids, min(4, new_tokens))  # warm-up
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
        torch.cuda.reset_peak_memory_stats(dev)
    if world > 1:
        dist.barrier()
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    t0 = time.time()
    sums = []
    tokens = greedy_generate(model, ids, new_tokens, sums)
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    dt = time.time() - t0
    peak = torch.cuda.max_memory_allocated(dev) / 2**20 if dev.type == "cuda" else 0.0
    t = torch.tensor([dt, peak], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0]), float(t[1]), tokens, torch.stack(sums)


def run(args):
    from .moe_ep import MoEConfig, Qwen3MoeEP, compress_ep_model, init_random
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.cpu:
        dev = torch.device("cpu")
        backend = "gloo"
    else:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        backend = "nccl"
    if world > 1:
        kw = {} if args.cpu else {"device_id": dev}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600), **kw)
    try:
        cfg = MoEConfig(num_hidden_layers=args.layers)
        if args.small:  # test-sized shape, same structure
            cfg = MoEConfig(vocab_size=256, hidden_size=128, num_hidden_layers=args.layers, num_attention_heads=4,
                            num_key_value_heads=2, head_dim=32, num_experts=8, num_experts_per_tok=2,
                            moe_intermediate_size=128)
        t0 = time.time()
        model = init_random(Qwen3MoeEP(cfg, rank, world, dev), args.seed)
        model.eval()
        build_s = time.time() - t0
        g = torch.Generator(device=dev).manual_seed(args.seed * 7919 + rank)
        ids = torch.randint(0, cfg.vocab_size, (args.batch, args.prompt_len), generator=g, device=dev)
        fp8 = sum(p.numel() for p in model.parameters() if p.dtype == torch.float8_e4m3fn)
        tu, pu, tok_u, sum_u = _timed(model, ids, args.new_tokens, world, dev)
        line = {
            "workload": f"config 5 generation: Qwen3-235B-A22B-shaped MoE, {cfg.num_hidden_layers} layers, "
                        f"{cfg.num_experts} experts top-{cfg.num_experts_per_tok}, expert-parallel x{world}, "
                        f"data-parallel attention",
            "n_gpus": world if not args.cpu else 0, "batch_per_rank": args.batch, "prompt_len": args.prompt_len,
            "new_tokens": args.new_tokens, "model_build_s": round(build_s, 1),
            "fp8_weights_per_rank": fp8,
            "uncompressed": {"latency_s": round(tu, 3), "tokens_per_s": round(args.batch * world * args.new_tokens / tu, 2),
                             "ms_per_step": round(tu / args.new_tokens * 1e3, 2), "peak_hbm_mb_max_rank": round(pu, 1)},
        }
        if not args.cpu:
            t1 = time.time()
            stream_bytes = compress_ep_model(model)
            torch.cuda.synchronize(dev)
            torch.cuda.empty_cache()
            line["compress_s"] = round(time.time() - t1, 1)
            line["ecf8_stream_bytes_per_rank"] = stream_bytes
            tc, pc, tok_c, sum_c = _timed(model, ids, args.new_tokens, world, dev)
            line["compressed"] = {"latency_s": round(tc, 3),
                                  "tokens_per_s": round(args.batch * world * args.new_tokens / tc, 2),
                                  "ms_per_step": round(tc / args.new_tokens * 1e3, 2),
                                  "peak_hbm_mb_max_rank": round(pc, 1)}
            same = torch.tensor([int(torch.equal(tok_u, tok_c)), int(torch.equal(sum_u, sum_c))], device=dev)
            if world > 1:
                dist.all_reduce(same, op=dist.ReduceOp.MIN)
            line["identical_tokens_all_ranks"] = bool(same[0])
            line["identical_logit_sums_all_ranks"] = bool(same[1])
            line["compressed_vs_uncompressed_tokens_per_s"] = round(tu / tc, 4)
        line["tokens"] = tok_u
        line["logit_sums"] = sum_u
        return rank, line
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


def main(argv=None):
    ap = argparse.ArgumentParser(description="Expert-parallel MoE generation, compressed vs uncompressed.")
    ap.add_argument("--layers", type=int, default=94)
    ap.add_argument("--batch", type=int, default=16, help="prompts per rank")
    ap.add_argument("--prompt_len", type=int, default=128)
    ap.add_argument("--new_tokens", type=int, default=32)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu", action="store_true", help="gloo + CPU tensors, uncompressed arm only")
    ap.add_argument("--small", action="store_true", help="test-sized dimensions")
    ap.add_argument("--out", type=str, default=None, help="write rank 0's tokens / logit sums here (torch.save)")
    args = ap.parse_args(argv)
    rank, line = run(args)
    if rank == 0:
        if args.out:
            torch.save({"tokens": line["tokens"].cpu(), "logit_sums": line["logit_sums"].cpu()}, args.out)
        line = {k: v for k, v in line.items() if k not in ("tokens", "logit_sums")}
        print(json.dumps(line), flush=True)
    return line


if __name__ == "__main__":
    main()
