#!/usr/bin/env python
"""ECF8 decode benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ecf8|reference]

N = 1 (default): config 2, the Qwen3-8B-shaped FP8 weight set: 36 layers,
each one ECF8 stream of q/k/v/o/gate/up/down (192,937,984 e4m3 weights,
sub-Linears concatenated in sorted-name order as the reference compressor
does), N(0, 0.02) weights with 128x128 block scales, seed layer*7 + index.
A step decodes every layer once into the per-device scratch buffer, one
C-ABI launch per layer, exactly as the decode-before-forward hook does.

N > 1 (under torchrun, one rank per GPU): config 5, the Qwen3-235B-A22B-shaped
MoE weight set.  Experts are partitioned evenly across ranks; each rank
decodes, per layer, its own experts plus its replica of the attention stream
with one batched launch.  No collective touches the data path.

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


def profiled_traffic(name):
    """Per-launch DRAM bytes recorded in profiles/<name> ("dram_bytes_per_launch: X")."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(p):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


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


def build_moe(dev, rank, world, n_layers):
    from ecf8_b200.codec import compress_fp8
    from ecf8_b200.run import build_decode_table
    per = QWEN3_235B_EXPERTS // world
    owned = list(range(rank * per, (rank + 1) * per))
    layers = []
    t0 = time.time()
    for l in range(n_layers):
        streams = [compress_fp8(make_stream_weights(QWEN3_235B_ATTN, (l * 1000 + 999) * 10, dev))]
        for e in owned:
            streams.append(compress_fp8(make_stream_weights(QWEN3_235B_EXPERT, (l * 1000 + e) * 10, dev)))
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


def run_ours(args, rank, world, dev):
    from ecf8_b200 import _lib
    from ecf8_b200.run import HostStreamDecoder, TensorManager, decode_streams
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    if world == 1:
        layers, originals = build_qwen3_8b(dev, args.layers)
        n_max = max(c["packed_other_4bits"].numel() * 2 for c in layers)
        scratch = TensorManager.get_tensor(dev, n_max).view(torch.uint8)
        calls = [decode_args(L, c, scratch, stream) for c in layers]
        elems = sum(c["packed_other_4bits"].numel() * 2 for c in layers)
        algo = sum(stream_bytes(c) for c in layers)
        launches_per_step = len(calls)

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
        launches_per_step = len(layers) * math.ceil(len(layers[0]) / 128)

        def step():
            for ly in layers:
                decode_streams(ly, outs, stream=stream, overlap_previous=True)

    # warm-up, then the timed region: K steps between a barrier + sync on both sides
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    n_launch_groups = len(calls) if world == 1 else len(layers)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        t_start.record(stream)
        for k in range(args.steps):
            step()
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms_total = t_start.elapsed_time(t_end)
    ms_step = max_over_ranks(ms_total / args.steps, world)
    # The timed region holds nothing but the decode launches, back to back
    # (each may overlap its set-up with the previous one's end), so the mean
    # launch duration is this rank's device time over its launches; no events
    # between launches, which would order them fully.
    mean_launch_ms = ms_total / (args.steps * n_launch_groups)

    # bit-exactness after timing
    exact = True
    if world == 1:
        for c, orig in zip(layers, originals):
            n = c["packed_other_4bits"].numel() * 2
            L.ecf8_decode_batch_flags(*decode_args(L, c, scratch, stream))
            exact &= bool(torch.equal(scratch[:n], orig))
    else:
        rng = np.random.default_rng(rank)
        for l in rng.choice(len(layers), size=min(3, len(layers)), replace=False):
            decode_streams(layers[l], outs, stream=stream)
            want = make_stream_weights(QWEN3_235B_ATTN, (int(l) * 1000 + 999) * 10, dev).view(torch.uint8)
            exact &= bool(torch.equal(outs[0], want))
            e = owned[len(owned) // 2]
            want = make_stream_weights(QWEN3_235B_EXPERT, (int(l) * 1000 + e) * 10, dev).view(torch.uint8)
            exact &= bool(torch.equal(outs[1 + len(owned) // 2], want))
    torch.cuda.synchronize()
    exact = max_over_ranks(0.0 if exact else 1.0, world) == 0.0

    total_elems = sum_over_ranks(elems, world)
    value = total_elems / (ms_step * 1e-3) / 1e9  # GB/s of e4m3 output, whole job
    peak, peak_kind = peak_hbm()
    # roofline of the dominant kernel: per-launch algorithmic bytes / mean launch time
    per_launch_bytes = algo / n_launch_groups
    achieved = per_launch_bytes / (mean_launch_ms * 1e-3) / 1e9
    traffic = profiled_traffic("decode_kernel_qwen3_8b_layer.md" if world == 1 else "none")

    # end to end through the host-buffer API: pinned host in, decode, pinned host out
    e2e = None
    if not args.no_e2e:
        if world == 1:
            e2e = run_e2e(args, layers, originals[-1], dev, world)
        else:  # a bounded sample of this rank's shard: its first two layers' streams
            sample = [s for ly in layers[:2] for s in ly]
            l_last = min(2, len(layers)) - 1
            want = make_stream_weights(QWEN3_235B_EXPERT, (l_last * 1000 + owned[-1]) * 10, dev).view(torch.uint8)
            e2e = run_e2e(args, sample, want, dev, world)
            e2e["sample"] = f"first {l_last + 1} layers of each rank's shard (attention + {len(owned)} experts each)"

    cpu = cpu_baseline(layers[0]) if (world == 1 and rank == 0 and not args.no_cpu_baseline) else None
    if rank != 0:
        return None
    cfg = {
        "workload": (f"config 2: Qwen3-8B-shaped FP8 weight set decode, {len(layers)} layer streams x 192,937,984 "
                     "e4m3 weights, one launch per layer into the shared scratch" if world == 1 else
                     f"config 5: Qwen3-235B-A22B-shaped MoE decode, {args.moe_layers} layers, 128 experts "
                     f"x 18,874,368 weights split {QWEN3_235B_EXPERTS // world}/GPU + attention replica "
                     "(71,303,168) per GPU, one batched launch per layer"),
        "elements_per_step": int(total_elems),
        "algorithmic_bytes_per_step_per_gpu": int(algo),
        "bytes_per_element": algo / elems,
        "l2": "inputs larger than L2 (no flush needed): "
              f"{algo / 2 ** 30:.2f} GiB touched per step per GPU vs 126 MiB L2",
        "weights": "N(0,0.02), 128x128 block scales absmax->448, e4m3fn; seeded per Linear",
        "decode_tables": "prepared once per stream at load (ecf8_build_table), 80 KB each",
        "parallelism": f"expert-sharded x{world}, no data-path collective" if world > 1 else "single GPU",
        "bit_exact": exact,
    }
    if world == 1:
        cfg["compressed_bits_per_element"] = sum(
            (c["encoded"].numel() + c["packed_other_4bits"].numel()) * 8 for c in layers) / elems
    line = {
        "metric": "ECF8 decode GB/s (fp8 out)",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak" if world == 1 else "strong",
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
            "kernel": "decode_kernel<128> (ecf8_decode_batch_flags launch, ECF8_DECODE_OVERLAP_PREVIOUS)",
            "algorithmic_bytes_per_launch": int(per_launch_bytes),
            "mean_launch_us": round(mean_launch_ms * 1e3, 2),
        },
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
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

def run_reference(args):
    """The reference decode on the host cores: the oracle's C restatement of
    dfloat/run/decode.cu (the reference has no CPU decoder), on layer 0 of the
    config-2 weight set, code table from the reference's Huffman dependency
    (restated) and LUTs / stream from restatements of its codec."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from dahuffman import HuffmanCodec
    t0 = time.time()
    parts = []
    for k, (_, o, i) in enumerate(QWEN3_8B_LINEARS):
        g = torch.Generator().manual_seed(k)
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
    s = {"luts": luts, "encoded": enc, "packed": packed, "gaps": gaps, "output_positions": op}
    log(f"reference arm: built layer-0 sample in {time.time() - t0:.1f}s")
    n = fp8.size
    out = np.empty(n, np.uint8)
    t1 = time.perf_counter()
    oracle.decode(s, out=out)
    first = time.perf_counter() - t1
    assert np.array_equal(out, fp8), "oracle decode is not bit-exact"
    # keep the whole run within a few minutes: shrink the sample to a prefix of groups
    budget = 150.0 / max(1, args.steps + args.warmup)
    if first > budget:
        groups = max(1, int((op.size - 1) * budget / first))
        end = int(op[groups])
        s = {"luts": luts, "encoded": enc[:groups * 4096], "packed": packed[:end // 2],
             "gaps": gaps[:groups * 256], "output_positions": np.concatenate([op[:groups], [end]]).astype(np.uint64)}
        n = end
        out = np.empty(n, np.uint8)
    for _ in range(args.warmup):
        oracle.decode(s, out=out)
    times = []
    for _ in range(args.steps):
        t1 = time.perf_counter()
        oracle.decode(s, out=out)
        times.append(time.perf_counter() - t1)
    dt = statistics.mean(times)
    value = n / dt / 1e9
    cores = oracle.max_threads()
    line = {
        "metric": "ECF8 decode GB/s (fp8 out)", "value": round(value, 3), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded random-init weights of the named shapes)",
        "config": {"workload": "config 2 sample: layer 0 of the Qwen3-8B-shaped weight set"
                               f" ({n:,} e4m3 weights per step)"},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{n:,} weights per step, C restatement of dfloat/run/decode.cu "
                                   "(the reference ships no CPU decoder), OpenMP over groups"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_gpu_kernel": reference_gpu_kernel(oracle, s, n, fp8[:n], args),
    }
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
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ecf8", "reference"], default="ecf8")
    ap.add_argument("--moe-layers", type=int, default=QWEN3_235B_LAYERS)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=QWEN3_8B_LAYERS,
                    help="config-2 layers to build (fewer only for profiling a small case)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    from ecf8_b200 import build
    build.build()
    try:
        line = run_ours(args, rank, world, dev)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
