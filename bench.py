#!/usr/bin/env python
"""ECF8 decode benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ecf8|reference]

Plain `python bench.py` (N = 1): config 2, the Qwen3-8B-shaped FP8 weight
set: 36 layers, each one ECF8 stream of q/k/v/o/gate/up/down (192,937,984
e4m3 weights, sub-Linears concatenated in sorted-name order as the reference
compressor does), N(0, 0.02) weights with 128x128 block scales, seed
layer*7 + index.  A step decodes every layer once into the per-device
scratch buffer, one C-ABI launch per layer, exactly as the
decode-before-forward hook does.

Under torchrun (one rank per GPU, any world size including 1): config 5, the
Qwen3-235B-A22B-shaped MoE weight set, --moe-layers layers (default 48, so
that the N = 1 shard fits one B200).  All 128 experts of every layer are
partitioned evenly across ranks; each rank decodes, per layer, its own
experts plus its replica of the attention stream with one batched launch.
No collective touches the data path.  The same workload at every N makes
the 1 -> 8 curve comparable.

--impl reference: the reference's CPU decode (the oracle's C restatement of
dfloat/run/decode.cu, all host threads) on a bounded sample of the same
workload, plus the reference kernel itself built for sm_100a on the GPU as an
extra field.  Rank 0 only.

One JSON line on stdout (rank 0).
"""

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

QWEN3_8B_LINEARS = [  # (name, out, in) in sorted-name order (flatten_block_of_weights)
    ("mlp.down_proj", 4096, 12288), ("mlp.gate_proj", 12288, 4096), ("mlp.up_proj", 12288, 4096),
    ("self_attn.k_proj", 1024, 4096), ("self_attn.o_proj", 4096, 4096),
    ("self_attn.q_proj", 4096, 4096), ("self_attn.v_proj", 1024, 4096),
]
QWEN3_8B_LAYERS = 36
QWEN3_235B_ATTN = [("k_proj", 512, 4096), ("o_proj", 4096, 8192), ("q_proj", 8192, 4096),
                   ("v_proj", 512, 4096)]
QWEN3_235B_EXPERT = [("down_proj", 4096, 1536), ("gate_proj", 1536, 4096), ("up_proj", 1536, 4096)]
QWEN3_235B_LAYERS = 94
QWEN3_235B_EXPERTS = 128
MOE_BENCH_LAYERS = 48  # config-5 layers a bench step decodes: the N = 1 shard (~104 GB) fits one B200
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 2 ** 20


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------
# Synthetic weights
# ---------------------------------------------------------------------------

def quantize_block128(w):
    o, i = w.shape
    t = w.reshape(o // 128, 128, i // 128, 128)
    amax = t.abs().amax(dim=(1, 3), keepdim=True).clamp(min=1e-12)
    return (t * (448.0 / amax)).to(torch.float8_e4m3fn).reshape(o, i)


def make_stream_weights(shapes, seed0, device):
    """Flat e4m3 block of the given Linear shapes; Linear k uses seed seed0 + k."""
    parts = []
    for k, (_, o, i) in enumerate(shapes):
        g = torch.Generator(device=device).manual_seed(seed0 + k)
        parts.append(quantize_block128(torch.randn(o, i, generator=g, device=device) * 0.02).reshape(-1))
    return torch.cat(parts)


def stream_bytes(c):
    """Algorithmic bytes of one decode: every stored buffer read once plus the
    e4m3 output written once."""
    n = c["packed_other_4bits"].numel() * 2
    table = c["decode_table"].numel() * c["decode_table"].element_size() if c.get("decode_table") is not None else 0
    return (c["encoded"].numel() + c["packed_other_4bits"].numel() + c["gaps"].numel()
            + c["output_positions"].numel() * 8 + c["luts"].numel() + table + n)


# ---------------------------------------------------------------------------
# Measurement helpers
# ---------------------------------------------------------------------------

class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index, period=0.002):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self.period, self.ok = period, False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report no clocks
            log("clock sampling unavailable:", e)

    def _run(self):
        nv = self.nv
        del nv
        while not self.stop:
            self.sample()
            time.sleep(self.period)

    def sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            pass

    def __enter__(self):
        if self.ok:
            self.sample()
            self.stop = False
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self.stop = True
            self.t.join()
            self.sample()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(name, per_launch_bytes):
    """DRAM bytes per launch from the ncu summary profiles/<name>: its
    captured launch's "dram_bytes_per_launch" scaled by this bench's
    algorithmic bytes per launch over the captured launch's
    ("algorithmic_bytes_per_launch"; the decode's traffic grows in proportion
    to the bytes it decodes).  None without a summary."""
    p = os.path.join(ROOT, "profiles", name)
    vals = {}
    try:
        for line in open(p):
            k, _, v = line.strip().partition(":")
            if k in ("dram_bytes_per_launch", "algorithmic_bytes_per_launch") and v.strip():
                vals[k] = float(v.split()[0])
    except OSError:
        return None
    if "dram_bytes_per_launch" not in vals:
        return None
    if "algorithmic_bytes_per_launch" not in vals:
        return vals["dram_bytes_per_launch"]
    return round(vals["dram_bytes_per_launch"] / vals["algorithmic_bytes_per_launch"] * per_launch_bytes)


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

def build_qwen3_8b(dev, n_layers=QWEN3_8B_LAYERS):
    from ecf8_b200.codec import compress_fp8
    from ecf8_b200.run import build_decode_table
    layers, originals = [], []
    t0 = time.time()
    for l in range(n_layers):
        flat = make_stream_weights(QWEN3_8B_LINEARS, l * 7, dev)
        c = compress_fp8(flat)
        c["decode_table"] = build_decode_table(c["luts"])  # once per stream, as at load time
        layers.append(c)
        originals.append(flat.view(torch.uint8))
    torch.cuda.synchronize()
    log(f"built {len(layers)} layer streams in {time.time() - t0:.1f}s")
    return layers, originals


def moe_plan(rank, world, n_layers):
    """Config-5 sharding: (owned experts, per-layer stream list) of one rank.
    Rank r owns experts [r * 128/N, (r+1) * 128/N) of every layer and a replica
    of the layer's attention stream; each stream is (name, seed of its first
    Linear, Linear shapes), the attention stream first."""
    if world < 1 or QWEN3_235B_EXPERTS % world:
        raise ValueError(f"{QWEN3_235B_EXPERTS} experts do not split evenly over {world} ranks")
    per = QWEN3_235B_EXPERTS // world
    owned = list(range(rank * per, (rank + 1) * per))
    layers = []
    for l in range(n_layers):
        ly = [(f"model.layers.{l}.self_attn", (l * 1000 + 999) * 10, QWEN3_235B_ATTN)]
        ly += [(f"model.layers.{l}.mlp.experts.{e}", (l * 1000 + e) * 10, QWEN3_235B_EXPERT) for e in owned]
        layers.append(ly)
    return owned, layers


def plan_elements(layers):
    return sum(o * i for ly in layers for _, _, shapes in ly for _, o, i in shapes)


def build_moe(dev, rank, world, n_layers):
    from ecf8_b200.codec import compress_fp8
    from ecf8_b200.run import build_decode_table
    owned, plan = moe_plan(rank, world, n_layers)
    layers = []
    t0 = time.time()
    for ly in plan:
        streams = [compress_fp8(make_stream_weights(shapes, seed, dev)) for _, seed, shapes in ly]
        for c in streams:
            c["decode_table"] = build_decode_table(c["luts"])
        layers.append(streams)
    torch.cuda.synchronize()
    log(f"rank {rank}: built {n_layers} layers x {len(owned)} experts + attention in {time.time() - t0:.1f}s")
    return layers, owned


def decode_args(L, c, out, stream):
    """ecf8_decode_batch_flags arguments for one stream with its prepared
    table: the launch the decode-before-forward hook makes once the table
    exists (it may start while the previous kernel finishes; the tables and
    streams were written at set-up, long before)."""
    from ecf8_b200 import _lib
    from ecf8_b200.run import _stream_struct
    arr = (_lib.Ecf8Stream * 1)(_stream_struct(c, out, c["decode_table"]))
    return (arr, 1, 512, 8, _lib.DECODE_OVERLAP_PREVIOUS, stream.cuda_stream)


def under_torchrun():
    """True when launched by torch.distributed.run (at any world size)."""
    return "TORCHELASTIC_RUN_ID" in os.environ or "LOCAL_WORLD_SIZE" in os.environ


def pick_workload(args):
    if args.workload != "auto":
        return args.workload
    return "config5" if under_torchrun() else "config2"


def timed_steps(step, k, stream, world, dev):
    """k steps between a barrier + synchronisation on both sides, timed with
    CUDA events on the launching stream; returns (ms per step, max over ranks;
    this rank's ms for all k steps; clock summary)."""
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        t_start.record(stream)
        for _ in range(k):
            step()
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms_total = t_start.elapsed_time(t_end)
    return max_over_ranks(ms_total / k, world), ms_total, clk.summary()


def call_convention_times(L, c, scratch, stream, reps=20):
    """Per-launch device time of one layer stream through three entry points,
    each launch ordered after the previous one (no overlap): the prepared
    table (what the hook passes), the reference's `_decode(grid=, block=,
    args=[...])` convention (its table cache built on the first call), and
    ecf8_decode without a table (every CTA derives it)."""
    from ecf8_b200 import _lib
    from ecf8_b200.run import _decode, _stream_struct
    n = c["packed_other_4bits"].numel() * 2
    arr = (_lib.Ecf8Stream * 1)(_stream_struct(c, scratch, c["decode_table"]))
    grid = (-(-c["encoded"].numel() // 4096),)
    ptrs = [c["luts"].data_ptr(), c["encoded"].data_ptr(), c["packed_other_4bits"].data_ptr(),
            c["output_positions"].data_ptr(), c["gaps"].data_ptr(), scratch.data_ptr()]
    n_op = c["output_positions"].numel()
    paths = {
        "prepared_table": lambda: L.ecf8_decode_batch(arr, 1, 512, 8, stream.cuda_stream),
        "reference_convention_decode": lambda: _decode(grid=grid, block=(512,), shared_mem=0,
                                                       args=ptrs + [c["luts"].shape[0], c["encoded"].numel(), n]),
        "no_table_ecf8_decode": lambda: L.ecf8_decode(*ptrs, c["luts"].shape[0], c["encoded"].numel(), n, n_op,
                                                      c["gaps"].numel(), 512, 8, stream.cuda_stream),
    }
    out = {}
    for name, fn in paths.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        out[name + "_us"] = round(a.elapsed_time(b) / reps * 1e3, 2)
    out["what"] = (f"one Qwen3-8B layer stream ({n:,} weights), {reps} launches each, ordered one after "
                   "another; _decode keeps one prepared table per LUT address")
    return out


def run_generation(args, dev):
    """Config 3, bounded: the full random-init Qwen3-8B architecture (36
    layers, FP8 Linears with 128x128 block scales), batch 16 x 128 random
    prompt ids, --gen-tokens greedy new tokens; the uncompressed FP8 model,
    then the same model with every decoder layer ECF8-compressed in place and
    decoded by the forward-pre-hook.  Each arm first runs one untimed
    generation of the same length; the timed one is between two
    synchronisations (inference_llm.py:109-160 of the reference).  Both arms
    use the same block-scaled FP8 GEMM, which reads e4m3 weights directly."""
    from ecf8_b200 import fp8_model
    from ecf8_b200.compress import compress_model_in_place
    from ecf8_b200.inference_llm import generate_timed, qwen3_8b_config
    from ecf8_b200.run import TensorManager
    t0 = time.time()
    model = fp8_model.fp8_model_from_config(qwen3_8b_config(QWEN3_8B_LAYERS), device=dev, seed=42)
    g = torch.Generator(device=dev).manual_seed(42)
    ids = torch.randint(0, model.config.vocab_size, (16, 128), generator=g, device=dev)
    n = args.gen_tokens
    unc, tok_u, sums_u, full_u = generate_timed(model, ids, n, keep=2, warm_tokens=n)
    compress_model_in_place(model)
    torch.cuda.synchronize()
    comp, tok_c, sums_c, full_c = generate_timed(model, ids, n, keep=2, warm_tokens=n)
    same = (bool(torch.equal(tok_u, tok_c)) and bool(torch.equal(sums_u, sums_c))
            and all(torch.equal(a, b) for a, b in zip(full_u, full_c)))
    out = {
        "workload": f"config 3 (bounded): Qwen3-8B architecture, 36 layers, batch 16 x 128 prompt ids, {n} greedy "
                    "new tokens, HF generate with the dynamic cache",
        "fp8_matmul": fp8_model.fp8_matmul_backend(),
        "uncompressed_tokens_per_s": round(unc["tokens_per_s"], 2),
        "compressed_tokens_per_s": round(comp["tokens_per_s"], 2),
        "compressed_vs_uncompressed": round(comp["tokens_per_s"] / unc["tokens_per_s"], 4),
        "uncompressed_ms_per_step": round(unc["ms_per_step"], 3),
        "compressed_ms_per_step": round(comp["ms_per_step"], 3),
        "peak_hbm_mb": {"uncompressed": round(unc["peak_hbm_mb"]), "compressed": round(comp["peak_hbm_mb"])},
        "identical_tokens_and_logits": same,
        "build_and_run_s": round(time.time() - t0, 1),
    }
    del model
    TensorManager.clear_device()
    return out


def run_ours(args, rank, world, dev):
    from ecf8_b200 import _lib
    from ecf8_b200.run import TensorManager, decode_streams
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    workload = pick_workload(args)
    if workload == "config2":
        if world > 1:
            raise SystemExit("config 2 is a one-GPU workload; run it without torchrun")
        layers, originals = build_qwen3_8b(dev, args.layers)
        n_max = max(c["packed_other_4bits"].numel() * 2 for c in layers)
        scratch = TensorManager.get_tensor(dev, n_max).view(torch.uint8)
        calls = [decode_args(L, c, scratch, stream) for c in layers]
        elems = sum(c["packed_other_4bits"].numel() * 2 for c in layers)
        algo = sum(stream_bytes(c) for c in layers)
        launches_per_step = len(calls)
        n_launch_groups = len(calls)

        def step():
            for a in calls:
                st = L.ecf8_decode_batch_flags(*a)
                if st:
                    raise RuntimeError(f"ecf8_decode_batch_flags failed: {st}")
    else:
        layers, owned = build_moe(dev, rank, world, args.moe_layers)
        per_layer = [s["packed_other_4bits"].numel() * 2 for s in layers[0]]
        outs = []
        off = 0
        scratch = torch.empty(sum(per_layer) + 16 * len(per_layer), dtype=torch.uint8, device=dev)
        for n in per_layer:
            outs.append(scratch[off:off + n])
            off += (n + 15) & ~15
        elems = sum(sum(s["packed_other_4bits"].numel() * 2 for s in ly) for ly in layers)
        algo = sum(sum(stream_bytes(s) for s in ly) for ly in layers)
        launches_per_step = len(layers) * math.ceil(len(layers[0]) / _lib.MAX_BATCH)
        n_launch_groups = launches_per_step

        def step():
            for ly in layers:
                decode_streams(ly, outs, stream=stream, overlap_previous=True)

    # warm-up, then the timed region: exactly K steps between a barrier + sync on both sides
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ms_step, ms_total, clocks = timed_steps(step, args.steps, stream, world, dev)
    # The timed region holds nothing but the decode launches, back to back
    # (each may overlap its set-up with the previous one's end), so the mean
    # launch duration is this rank's device time over its launches; no events
    # between launches, which would order them fully.
    mean_launch_ms = ms_total / (args.steps * n_launch_groups)

    # Steady state: at least --steady-s seconds of device time (same steps),
    # so that the clock samples see the kernel at its sustained clocks.
    steady = None
    if args.steady_s > 0:
        k2 = max(args.steps, math.ceil(args.steady_s * 1e3 / ms_step))
        ms2, total2, clk2 = timed_steps(step, k2, stream, world, dev)
        steady = {"steps": k2, "ms_per_step": round(ms2, 4), "device_s": round(total2 / 1e3, 3),
                  "mean_launch_us": round(total2 / (k2 * n_launch_groups) * 1e3, 2), "clocks": clk2}

    # bit-exactness after timing
    exact = True
    if workload == "config2":
        for c, orig in zip(layers, originals):
            n = c["packed_other_4bits"].numel() * 2
            L.ecf8_decode_batch_flags(*decode_args(L, c, scratch, stream))
            exact &= bool(torch.equal(scratch[:n], orig))
    else:
        _, plan = moe_plan(rank, world, args.moe_layers)
        rng = np.random.default_rng(rank)
        for l in rng.choice(len(layers), size=min(3, len(layers)), replace=False):
            decode_streams(layers[l], outs, stream=stream)
            for j in (0, 1, len(owned) // 2, len(owned)):
                _, seed, shapes = plan[l][j]
                exact &= bool(torch.equal(outs[j], make_stream_weights(shapes, seed, dev).view(torch.uint8)))
    torch.cuda.synchronize()
    exact = max_over_ranks(0.0 if exact else 1.0, world) == 0.0

    total_elems = sum_over_ranks(elems, world)
    value = total_elems / (ms_step * 1e-3) / 1e9  # GB/s of e4m3 output, whole job
    peak, peak_kind = peak_hbm()
    # roofline of the dominant kernel: per-launch algorithmic bytes / mean launch time
    per_launch_bytes = algo / n_launch_groups
    achieved = per_launch_bytes / (mean_launch_ms * 1e-3) / 1e9
    traffic = profiled_traffic("decode_kernel_qwen3_8b_layer.md" if workload == "config2"
                               else "decode_kernel_config5_layer.md", per_launch_bytes)
    if steady is not None:
        steady["roofline_frac"] = round(per_launch_bytes / (steady["mean_launch_us"] * 1e-6) / 1e9 / peak, 4)
        steady["value"] = round(total_elems / (steady["ms_per_step"] * 1e-3) / 1e9, 2)

    # end to end through the host-buffer API: pinned host in, decode, pinned host out
    e2e = None
    if not args.no_e2e:
        if workload == "config2":
            e2e = run_e2e(args, layers, originals[-1], dev, world)
        else:  # a bounded sample of this rank's shard: its first two layers' streams
            _, plan = moe_plan(rank, world, args.moe_layers)
            sample = [s for ly in layers[:2] for s in ly]
            l_last = min(2, len(layers)) - 1
            _, seed, shapes = plan[l_last][-1]
            e2e = run_e2e(args, sample, make_stream_weights(shapes, seed, dev).view(torch.uint8), dev, world)
            e2e["sample"] = f"first {l_last + 1} layers of each rank's shard (attention + {len(owned)} experts each)"

    conv = None
    if workload == "config2" and not args.no_call_conventions:
        conv = call_convention_times(L, layers[0], scratch, stream)
    gen = None
    if workload == "config2" and args.gen_tokens > 0:
        del calls, scratch
        torch.cuda.empty_cache()
        gen = run_generation(args, dev)
    cpu = cpu_baseline(layers[0]) if (workload == "config2" and rank == 0 and not args.no_cpu_baseline) else None
    if rank != 0:
        return None
    if workload == "config2":
        cfg = {
            "workload": (f"config 2: Qwen3-8B-shaped FP8 weight set decode, {len(layers)} layer streams x "
                         "192,937,984 e4m3 weights, one launch per layer into the shared scratch"),
            "parallelism": "single GPU",
            "compressed_bits_per_element": sum(
                (c["encoded"].numel() + c["packed_other_4bits"].numel()) * 8 for c in layers) / elems,
        }
    else:
        cfg = {
            "workload": (f"config 5: Qwen3-235B-A22B-shaped MoE decode, {args.moe_layers} layers, 128 experts "
                         f"x 18,874,368 weights split {QWEN3_235B_EXPERTS // world}/GPU + attention replica "
                         "(71,303,168) per GPU, one batched launch per layer (up to 256 streams per launch)"),
            "parallelism": f"expert-sharded x{world}, no data-path collective",
            "scaling_note": ("all 128 experts of every layer are split over the ranks (fixed total); each rank "
                             "also decodes a replica of the attention stream, counted in value"),
        }
    cfg.update({
        "elements_per_step": int(total_elems),
        "algorithmic_bytes_per_step_per_gpu": int(algo),
        "bytes_per_element": algo / elems,
        "l2": "inputs larger than L2 (no flush needed): "
              f"{algo / 2 ** 30:.2f} GiB touched per step per GPU vs 126 MiB L2",
        "weights": "N(0,0.02), 128x128 block scales absmax->448, e4m3fn; seeded per Linear",
        "decode_tables": f"prepared once per stream at load (ecf8_build_table), {_lib.TABLE_BYTES} B each",
        "bit_exact": exact,
    })
    line = {
        "metric": "ECF8 decode GB/s (fp8 out)",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak" if workload == "config2" else "strong",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic (seeded random-init weights of the named shapes)",
        "config": cfg,
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": traffic,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
            else "fallback 6.65 TB/s",
            "kernel": f"decode_kernel<{_lib.MAX_BATCH}> (ecf8_decode_batch_flags launch, "
                      "ECF8_DECODE_OVERLAP_PREVIOUS)",
            "algorithmic_bytes_per_launch": int(per_launch_bytes),
            "mean_launch_us": round(mean_launch_ms * 1e3, 2),
        },
        "steady_state": steady,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if conv is not None:
        line["call_conventions"] = conv
    if gen is not None:
        line["generation"] = gen
    return line


def run_e2e(args, layers, last_original, dev, world):
    """Same metric through HostStreamDecoder: each step copies every stream's
    buffers from pinned host memory, decodes, and copies the e4m3 weights
    back to pinned host memory.  Under torchrun every rank does this for its
    own streams between a barrier and a synchronisation; the step time is the
    maximum over ranks and the elements are summed over ranks."""
    from ecf8_b200.run import STREAM_BUFFERS, HostStreamDecoder
    host = []
    for c in layers:
        h = {}
        for k in STREAM_BUFFERS:
            t = c[k]
            p = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            p.copy_(t)
            h[k] = p
        host.append(h)
    n_max = max(c["packed_other_4bits"].numel() * 2 for c in layers)
    ring = [torch.empty(n_max, dtype=torch.uint8, pin_memory=True) for _ in range(4)]
    outs = [ring[i % len(ring)][:c["packed_other_4bits"].numel() * 2] for i, c in enumerate(layers)]
    dec = HostStreamDecoder(dev, depth=2)
    tables = [c["decode_table"] for c in layers]
    dec.decode(host, outs, tables)  # warm-up: staging slots grow to their largest stream here
    steps = max(1, min(args.steps, args.e2e_steps))
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        dec.decode(host, outs, tables)
    torch.cuda.synchronize()
    dt = max_over_ranks((time.perf_counter() - t0) / steps, world)
    elems = sum_over_ranks(sum(c["packed_other_4bits"].numel() * 2 for c in layers), world)
    h2d = sum_over_ranks(sum(sum(h[k].numel() * h[k].element_size() for k in STREAM_BUFFERS) for h in host), world)
    exact = bool(torch.equal(outs[-1], last_original.cpu()))
    exact = max_over_ranks(0.0 if exact else 1.0, world) == 0.0
    return {"value": round(elems / dt / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
            "bit_exact": exact,
            "d2h_bytes_per_step": int(elems), "steps": steps, "ms_per_step": round(dt * 1e3, 2),
            "api": "ecf8_b200.run.HostStreamDecoder (pinned host buffers, C-ABI decode)"}


def host_stream(c):
    return {"luts": c["luts"].cpu().numpy(), "encoded": c["encoded"].cpu().numpy(),
            "packed": c["packed_other_4bits"].cpu().numpy(), "gaps": c["gaps"].cpu().numpy(),
            "output_positions": c["output_positions"].view(torch.int64).cpu().numpy().view(np.uint64)}


def cpu_baseline(c, budget_s=10.0):
    """The oracle (C restatement of the reference decode kernel) on all host
    threads, decoding layer 0 repeatedly for about `budget_s` seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    s = host_stream(c)
    n = s["packed"].size * 2
    out = np.empty(n, np.uint8)
    oracle.decode(s, out=out)
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.decode(s, out=out)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(n / dt / 1e9, 3), "unit": "GB/s", "cores": oracle.max_threads(), "kind": "port",
            "sample": f"layer 0 of the Qwen3-8B-shaped set ({n:,} weights) decoded {reps}x by the C "
                      "restatement of dfloat/run/decode.cu on all host threads (OpenMP over groups)"}


# ---------------------------------------------------------------------------
# Reference arm
# ---------------------------------------------------------------------------

def reference_sample_streams(oracle, workload):
    """The reference arm's sample of the bench workload, as host streams built
    with the restated reference codec: config 2 -> layer 0 (one stream);
    config 5 -> layer 0's attention stream and its first four experts."""
    from dahuffman import HuffmanCodec
    if workload == "config2":
        groups = [(QWEN3_8B_LINEARS, 0)]
    else:
        _, plan = moe_plan(0, 1, 1)
        groups = [(shapes, seed) for _, seed, shapes in plan[0][:5]]
    out = []
    for shapes, seed0 in groups:
        parts = []
        for k, (_, o, i) in enumerate(shapes):
            g = torch.Generator().manual_seed(seed0 + k)
            parts.append(quantize_block128(torch.randn(o, i, generator=g) * 0.02).reshape(-1))
        fp8 = torch.cat(parts).view(torch.uint8).numpy()
        e, packed = oracle.split(fp8)
        cnt = np.bincount(e, minlength=16)
        codec = HuffmanCodec.from_frequencies({s: int(c) for s, c in enumerate(cnt) if c})
        table = codec.get_code_table()
        bits = np.zeros(16, np.uint8)
        vals = np.zeros(16, np.uint32)
        for s, (b, v) in table.items():
            if isinstance(s, int):
                bits[s], vals[s] = b, v
        eb, ev = table[codec._eof]
        luts = oracle.luts_from_table(table)
        enc, gaps, op = oracle.encode(e, bits, vals, eb, ev)
        out.append(({"luts": luts, "encoded": enc, "packed": packed, "gaps": gaps, "output_positions": op}, fp8))
    return out


def run_reference(args):
    """The reference decode on the host cores: the oracle's C restatement of
    dfloat/run/decode.cu (the reference has no CPU decoder), on a sample of the
    bench's own workload (config 2, or config 5 under torchrun), code tables
    from the reference's Huffman dependency (restated) and LUTs / streams from
    restatements of its codec.  A step decodes every sample stream once."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    workload = pick_workload(args)
    t0 = time.time()
    sample = reference_sample_streams(oracle, workload)
    log(f"reference arm: built the {workload} sample in {time.time() - t0:.1f}s")
    outs = [np.empty(fp8.size, np.uint8) for _, fp8 in sample]
    t1 = time.perf_counter()
    for (s, fp8), out in zip(sample, outs):
        oracle.decode(s, out=out)
        assert np.array_equal(out, fp8), "oracle decode is not bit-exact"
    first = time.perf_counter() - t1
    # keep the whole run within a few minutes: shrink each stream to a prefix of groups
    budget = 150.0 / max(1, args.steps + args.warmup)
    if first > budget:
        frac = budget / first
        cut = []
        for s, fp8 in sample:
            op = s["output_positions"]
            groups = max(1, int((op.size - 1) * frac))
            end = int(op[groups])
            cut.append(({"luts": s["luts"], "encoded": s["encoded"][:groups * 4096], "packed": s["packed"][:end // 2],
                         "gaps": s["gaps"][:groups * 256],
                         "output_positions": np.concatenate([op[:groups], [end]]).astype(np.uint64)}, fp8[:end]))
        sample = cut
        outs = [np.empty(fp8.size, np.uint8) for _, fp8 in sample]
    n = sum(fp8.size for _, fp8 in sample)

    def step():
        for (s, _), out in zip(sample, outs):
            oracle.decode(s, out=out)
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t1 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t1)
    dt = statistics.mean(times)
    value = n / dt / 1e9
    cores = oracle.max_threads()
    what = ("config 2 sample: layer 0 of the Qwen3-8B-shaped weight set" if workload == "config2" else
            "config 5 sample: layer 0 attention stream + experts 0-3 of the Qwen3-235B-A22B-shaped set")
    line = {
        "metric": "ECF8 decode GB/s (fp8 out)", "value": round(value, 3), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded random-init weights of the named shapes)",
        "config": {"workload": f"{what} ({n:,} e4m3 weights per step)"},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{n:,} weights per step, C restatement of dfloat/run/decode.cu "
                                   "(the reference ships no CPU decoder), OpenMP over groups"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if workload == "config2":
        s, fp8 = sample[0]
        line["reference_gpu_kernel"] = reference_gpu_kernel(oracle, s, fp8.size, fp8, args)
    return line


def reference_gpu_kernel(oracle, s, n, want, args):
    """The reference kernel decode.cu compiled unmodified for sm_100a
    (oracle/_ref), launched with the reference geometry on the same sample."""
    if not torch.cuda.is_available():
        return None
    if not os.path.exists(oracle.REF_LIB):
        return {"unavailable": "oracle/_ref/libref_decode.so was not built (no reference checkout)"}
    if not oracle.reference_kernel_terminates(s["luts"]):
        return {"unavailable": "this sample's LUTs contain a length-0 path; the reference kernel would spin"}
    dev = torch.device("cuda", 0)
    luts = np.zeros((18, 256), np.uint8)
    luts[:s["luts"].shape[0]] = s["luts"]
    op = np.concatenate([s["output_positions"], [np.uint64(n)]]).astype(np.uint64)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dl, de, dp, do, dg = t(luts), t(s["encoded"]), t(s["packed"]), t(op.view(np.int64)), t(s["gaps"])
    out = torch.empty(n, dtype=torch.uint8, device=dev)
    grid = math.ceil(s["encoded"].size / 4096)
    smem = 512 * 4 + 4 + int(np.diff(s["output_positions"].astype(np.int64)).max())
    L = oracle.ref_lib()
    st = torch.cuda.current_stream(dev)

    def launch():
        r = L.ref_decode_launch(dl.data_ptr(), de.data_ptr(), dp.data_ptr(), do.data_ptr(), dg.data_ptr(),
                                out.data_ptr(), s["luts"].shape[0], s["encoded"].size, n, grid, 512, smem,
                                st.cuda_stream)
        if r:
            raise RuntimeError(f"reference kernel launch failed: {r}")
    for _ in range(max(args.warmup, 3)):
        launch()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(args.steps, 10)
    a.record(st)
    for _ in range(reps):
        launch()
    b.record(st)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    exact = bool(np.array_equal(out.cpu().numpy(), want))
    algo = s["encoded"].size + s["packed"].size + s["gaps"].size + op.size * 8 + s["luts"].size + n
    peak, _ = peak_hbm()
    return {"value": round(n / (ms * 1e-3) / 1e9, 2), "unit": "GB/s (fp8 out)", "ms_per_launch": round(ms, 4),
            "bit_exact": exact,
            "hbm_frac": round(algo / (ms * 1e-3) / 1e9 / peak, 4),
            "what": "reference dfloat/run/decode.cu built for sm_100a, one launch per layer-0 sample"}


# ---------------------------------------------------------------------------

def main():
    # Stdout carries the one JSON line only: whatever libraries print there
    # (NCCL's version banner at communicator creation, for one) goes to stderr.
    out_fd = os.dup(1)
    os.dup2(2, 1)
    try:
        line = _main()
    finally:
        sys.stdout.flush()
        os.dup2(out_fd, 1)
        os.close(out_fd)
    if line is not None:
        print(json.dumps(line), flush=True)


def _main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ecf8", "reference"], default="ecf8")
    ap.add_argument("--moe-layers", type=int, default=MOE_BENCH_LAYERS)
    ap.add_argument("--workload", choices=["auto", "config2", "config5"], default="auto",
                    help="auto: config 5 under torchrun (any world size), config 2 otherwise")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--steady-s", type=float, default=1.0,
                    help="device seconds of the steady-state measurement after the K timed steps (0: off)")
    ap.add_argument("--no-call-conventions", action="store_true")
    ap.add_argument("--gen-tokens", type=int, default=64,
                    help="config-3 generation measured after the decode bench (new tokens per arm; 0: off)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=QWEN3_8B_LAYERS,
                    help="config-2 layers to build (fewer only for profiling a small case)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args) if rank == 0 else None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if under_torchrun():
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    from ecf8_b200 import build
    build.build()
    try:
        line = run_ours(args, rank, world, dev)
    finally:
        if under_torchrun():
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
    return line if rank == 0 else None


if __name__ == "__main__":
    main()
