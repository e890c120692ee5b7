"""DiT denoising with on-the-fly ECF8 decode, compressed vs uncompressed
(config 4; stands in for the reference's scripts/inference_dfsyn.py FLUX
runs, whose pipeline package and prompts are not available here).

    python -m ecf8_b200.inference_dit

One 1024x1024 image: 4096 image tokens of 64 latent channels (a 128x128x16
latent patchified 2x2), 512 text tokens of N(0, 1) 4096-d embeddings, a
pooled 768-d text vector, guidance 3.5, 28 Euler flow-matching steps on a
linear sigma schedule.  Both arms run in one process on one model: first
uncompressed, then with every `dit.blocks.N` / `dit.single_blocks.N` stream
decoded in its forward-pre-hook.  Each arm is warmed up by a few steps, then
every step is timed with CUDA events; the final latents and every step's
velocity (float64 sum) must be bit-identical between the arms.
"""

import argparse
import json
import time

import torch


def denoise(pipe, latents, text, pooled, cos, sin, steps=28, guidance=3.5, warm=3):
    dev = latents.device
    sig = torch.linspace(1.0, 0.0, steps + 1, device=dev)
    g = torch.full((1,), guidance, device=dev)
    x = latents.float()
    with torch.no_grad():
        for i in range(warm):  # warm-up steps, not part of the trajectory
            pipe.dit(x.to(torch.bfloat16), text, pooled, sig[i:i + 1], g, cos, sin)
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        sums = []
        t0 = time.time()
        for i in range(steps):
            ev[i][0].record()
            v = pipe.dit(x.to(torch.bfloat16), text, pooled, sig[i:i + 1], g, cos, sin)
            x = x + (sig[i + 1] - sig[i]) * v.float()
            ev[i][1].record()
            sums.append(v.double().sum())
        torch.cuda.synchronize()
        wall = time.time() - t0
    ms = [a.elapsed_time(b) for a, b in ev]
    return {"ms_per_step": sum(ms) / steps, "min_ms_per_step": min(ms), "max_ms_per_step": max(ms),
            "total_s": wall, "peak_hbm_mb": torch.cuda.max_memory_allocated() / 2**20}, x, torch.stack(sums)


def main(argv=None):
    ap = argparse.ArgumentParser(description="Compressed vs uncompressed FLUX-shaped DiT denoising (config 4).")
    ap.add_argument("--steps", type=int, default=28)
    ap.add_argument("--warm", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--n_double", type=int, default=19)
    ap.add_argument("--n_single", type=int, default=38)
    ap.add_argument("--image_tokens", type=int, default=4096, help="a square number")
    ap.add_argument("--text_tokens", type=int, default=512)
    args = ap.parse_args(argv)
    from .compress import compress_model_in_place
    from .dit_model import flux_dit_pipeline, position_ids, rope_freqs
    from .run import TensorManager
    dev = torch.device("cuda", torch.cuda.current_device())
    t0 = time.time()
    pipe = flux_dit_pipeline(device=dev, seed=args.seed, n_double=args.n_double, n_single=args.n_single)
    build_s = time.time() - t0
    gen = torch.Generator(device=dev).manual_seed(args.seed + 12345)
    side = int(round(args.image_tokens ** 0.5))
    latents = torch.randn(1, side * side, 64, generator=gen, device=dev)
    text = torch.randn(1, args.text_tokens, 4096, generator=gen, device=dev).to(torch.bfloat16)
    pooled = torch.randn(1, 768, generator=gen, device=dev).to(torch.bfloat16)
    cos, sin = rope_freqs(position_ids(args.text_tokens, side, side, dev))
    fp8 = sum(p.numel() for p in pipe.parameters() if p.dtype == torch.float8_e4m3fn)
    line = {"workload": f"config 4: FLUX.1-dev-shaped DiT ({args.n_double} double + {args.n_single} single "
                        f"blocks, hidden 3072), {side * side} image + {args.text_tokens} text tokens, "
                        f"{args.steps} steps", "model_build_s": round(build_s, 1), "fp8_weights": fp8}
    res_u, x_u, s_u = denoise(pipe, latents, text, pooled, cos, sin, args.steps, warm=args.warm)
    line["uncompressed"] = {k: round(v, 3) for k, v in res_u.items()}
    t1 = time.time()
    compress_model_in_place(pipe)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    TensorManager.clear_device()
    line["compress_s"] = round(time.time() - t1, 1)
    line["ecf8_stream_bytes"] = sum(b.numel() * b.element_size() for m in pipe.modules()
                                    for k, b in m._buffers.items()
                                    if k in ("luts", "encoded", "packed_other_4bits", "output_positions", "gaps"))
    res_c, x_c, s_c = denoise(pipe, latents, text, pooled, cos, sin, args.steps, warm=args.warm)
    line["compressed"] = {k: round(v, 3) for k, v in res_c.items()}
    line["finite_output"] = bool(torch.isfinite(x_u).all())
    line["identical_latents"] = bool(torch.equal(x_u, x_c))
    line["identical_velocity_sums_all_steps"] = bool(torch.equal(s_u, s_c))
    line["compressed_vs_uncompressed_step_latency"] = round(res_c["ms_per_step"] / res_u["ms_per_step"], 4)
    print(json.dumps(line), flush=True)
    return line


if __name__ == "__main__":
    main()
