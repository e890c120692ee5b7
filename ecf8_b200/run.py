"""Runtime integration: per-device scratch, decode-before-forward hook, loaders.

Mirrors the public surface of zeyuyang8/ecf8 ``dfloat.run``
(dfloat/run/__init__.py:1-17, dfloat/run/run.py) with the same names,
arguments, buffer names and on-disk layout; the decode itself goes through
the C ABI of libecf8_b200.so (include/ecf8.h) on PyTorch's current stream.

  TensorManager                       run.py:36-81
  get_hook                            run.py:84-155
  _decode (kernel-launch drop-in)     run.py:24-33, call sites run.py:103-119,
                                      scripts/compress.py:109-124
  load_and_replace_tensors            run.py:158-275
  load_and_replace_tensors_parallel   run.py:278-403 (+ 406-458)
  get_dfloat_model_name_or_path       run.py:473-480
  DFloatModel.from_pretrained         run.py:483-566
  DFloatDiffSynthModelFP8             run.py:569-729
"""

import json
import math
import os
import re
import threading
from collections import OrderedDict
from sys import stderr
from typing import Dict, Optional, Union

import torch
import torch.nn as nn

from . import _lib
from .const import get_default_no_split_pattern

STREAM_BUFFERS = ("luts", "encoded", "packed_other_4bits", "output_positions", "gaps")


# ---------------------------------------------------------------------------
# Scratch
# ---------------------------------------------------------------------------

class TensorManager:
    """One grow-only e4m3 buffer per device; every hooked block decodes into
    a prefix of it, so only the largest block's decoded weights are resident
    at a time (run.py:36-81)."""

    _tensors = {}
    _lock = threading.Lock()

    @staticmethod
    def get_tensor(device, n_elements, dtype=torch.float8_e4m3fn):
        if isinstance(device, str):
            device = torch.device(device)
        with TensorManager._lock:
            cur = TensorManager._tensors.get(device)
            if cur is not None and cur.numel() >= n_elements and cur.dtype == dtype:
                return cur[:n_elements]
            if cur is not None:
                del TensorManager._tensors[device]
                del cur
                torch.cuda.empty_cache()
            new = torch.empty(n_elements, dtype=dtype, device=device)
            print(f"Allocated {n_elements} {dtype} on device {device}", file=stderr)
            TensorManager._tensors[device] = new
            return new

    @staticmethod
    def clear_device(device=None):
        with TensorManager._lock:
            if device is None:
                TensorManager._tensors.clear()
            else:
                if isinstance(device, str):
                    device = torch.device(device)
                TensorManager._tensors.pop(device, None)
        torch.cuda.empty_cache()


# ---------------------------------------------------------------------------
# Decode entry points
# ---------------------------------------------------------------------------

def _check_u8(t, name, device):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def build_decode_table(luts, stream=None):
    """The stream's multi-symbol decode table (_lib.TABLE_BYTES as an int32 tensor on the
    LUTs' device), derived from its LUTs by ecf8_build_table.  It depends on
    the LUTs only: build it once per stream and pass it to every decode."""
    device = luts.device
    _check_u8(luts, "luts", device)
    if device.type != "cuda":
        raise ValueError("the decode table is built on a CUDA device")
    table = torch.empty(_lib.TABLE_BYTES // 4, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        s = stream if stream is not None else torch.cuda.current_stream(device)
        st = _lib.lib().ecf8_build_table(luts.data_ptr(), luts.shape[0], table.data_ptr(), s.cuda_stream)
    _lib.check(st, "ecf8_build_table")
    return table


def _stream_struct(s, out, table=None):
    n = s["packed_other_4bits"].numel() * 2
    return _lib.Ecf8Stream(
        s["luts"].data_ptr(), s["luts"].shape[0], 0, s["encoded"].data_ptr(), s["encoded"].numel(),
        s["packed_other_4bits"].data_ptr(), s["output_positions"].data_ptr(),
        s["output_positions"].numel() * s["output_positions"].element_size() // 8,
        s["gaps"].data_ptr(), s["gaps"].numel() * s["gaps"].element_size(), out.data_ptr(), n,
        table.data_ptr() if table is not None else None)


def _check_stream(s, out, device, table=None):
    for name in STREAM_BUFFERS:
        _check_u8(s[name], name, device)
    _check_u8(out, "out", device)
    if s["luts"].dim() != 2 or s["luts"].shape[1] != 256:
        raise ValueError("luts must have shape (n_luts, 256)")
    n = s["packed_other_4bits"].numel() * 2
    if out.numel() * out.element_size() < n:
        raise ValueError(f"out holds {out.numel() * out.element_size()} bytes, the stream has {n} elements")
    if table is not None:
        _check_u8(table, "table", device)
        if table.numel() * table.element_size() != _lib.TABLE_BYTES:
            raise ValueError(f"a decode table has {_lib.TABLE_BYTES} bytes")


def decode_stream(luts, encoded, packed_other_4bits, output_positions, gaps, out=None,
                  threads_per_block=512, bytes_per_thread=8, stream=None, table=None, overlap_previous=False,
                  max_ctas=0):
    """Decodes one ECF8 stream (the five buffers a compressed block holds) into
    `out` (e4m3 or uint8, n = 2 * packed_other_4bits.numel() elements;
    allocated if None).  `table` is the stream's prepared decode table
    (build_decode_table), or None to derive it inside the kernel.
    Asynchronous on `stream` (default: the current stream of the buffers'
    device).  With overlap_previous=True the launch may start while the
    stream's previous kernel runs and writes `out` only after it has finished
    (ECF8_DECODE_OVERLAP_PREVIOUS); the caller guarantees that no work still
    in flight on the stream writes the stream buffers or the table.  With
    max_ctas > 0 the launch uses at most that many CTAs (ECF8_DECODE_CTAS)
    instead of one per SM, leaving the other SMs to kernels on other streams.
    Returns `out`."""
    device = encoded.device
    if device.type != "cuda":
        raise ValueError("ECF8 decode runs on a CUDA device; move the stream buffers there first")
    n = packed_other_4bits.numel() * 2
    if out is None:
        out = torch.empty(n, dtype=torch.float8_e4m3fn, device=device)
    s = {"luts": luts, "encoded": encoded, "packed_other_4bits": packed_other_4bits,
         "output_positions": output_positions, "gaps": gaps}
    _check_stream(s, out, device, table)
    L = _lib.lib()
    with torch.cuda.device(device):
        cs = stream if stream is not None else torch.cuda.current_stream(device)
        if overlap_previous or max_ctas:
            flags = (_lib.DECODE_OVERLAP_PREVIOUS if overlap_previous else 0) | \
                (_lib.decode_ctas(max_ctas) if max_ctas else 0)
            arr = (_lib.Ecf8Stream * 1)(_stream_struct(s, out, table))
            st = L.ecf8_decode_batch_flags(arr, 1, threads_per_block, bytes_per_thread, flags, cs.cuda_stream)
        elif table is None:
            st = L.ecf8_decode(luts.data_ptr(), encoded.data_ptr(), packed_other_4bits.data_ptr(),
                               output_positions.data_ptr(), gaps.data_ptr(), out.data_ptr(),
                               luts.shape[0], encoded.numel(), n,
                               output_positions.numel() * output_positions.element_size() // 8,
                               gaps.numel() * gaps.element_size(), threads_per_block, bytes_per_thread,
                               cs.cuda_stream)
        else:
            arr = (_lib.Ecf8Stream * 1)(_stream_struct(s, out, table))
            st = L.ecf8_decode_batch(arr, 1, threads_per_block, bytes_per_thread, cs.cuda_stream)
    _lib.check(st, "ecf8_decode")
    return out


def decode_streams(streams, outs, threads_per_block=512, bytes_per_thread=8, stream=None,
                   overlap_previous=False):
    """Decodes several streams with one persistent launch per 256 streams.
    `streams` is a list of dicts with the five stream buffers (and optionally
    "decode_table"); `outs` the matching output tensors.  All on one device.
    overlap_previous as in decode_stream."""
    if len(streams) != len(outs):
        raise ValueError("one output per stream")
    if not streams:
        return outs
    device = streams[0]["encoded"].device
    arr = (_lib.Ecf8Stream * len(streams))()
    for i, (s, o) in enumerate(zip(streams, outs)):
        table = s.get("decode_table")
        _check_stream(s, o, device, table)
        arr[i] = _stream_struct(s, o, table)
    L = _lib.lib()
    with torch.cuda.device(device):
        cs = stream if stream is not None else torch.cuda.current_stream(device)
        flags = _lib.DECODE_OVERLAP_PREVIOUS if overlap_previous else 0
        st = L.ecf8_decode_batch_flags(arr, len(streams), threads_per_block, bytes_per_thread, flags, cs.cuda_stream)
    _lib.check(st, "ecf8_decode_batch_flags")
    return outs


class _DecodeLauncher:
    """Drop-in for the reference's ``_decode`` CuPy RawKernel (run.py:29-33).

    Called like the reference launch: ``_decode(grid=(G,), block=(512,),
    shared_mem=S, args=[luts, encoded, packed_other_4bits, output_positions,
    gaps, outputs, n_luts, n_bytes, n_elements])`` where the six buffers are
    device pointers (ints) or tensors on the current device.  grid / block
    must be the reference geometry (G = ceil(n_bytes / 4096), 512 threads);
    shared_mem is accepted and ignored (the engine sizes its own).  Like the
    reference it launches asynchronously on the current stream and returns
    nothing; unlike it, a bad argument raises.  output_positions is read for
    the first G entries only (the trailing entry is always n_elements), so a
    short array is safe.

    The multi-symbol decode table is built once per (device, luts address,
    n_luts) and kept in a small cache (`cache_size` tables of
    ECF8_TABLE_BYTES each), so repeated calls on a block do not derive it in
    every CTA of every launch.  The kernel compares each cached table's copy
    of the LUTs with the LUTs it is given and derives the table itself when
    they differ, so a cached table whose LUT memory was reused for other LUTs
    only costs that derivation; ``clear_cache()`` drops every cached table.
    """

    bytes_per_thread = 8
    cache_size = 256

    def __init__(self):
        self._tables = OrderedDict()
        self._lock = threading.Lock()

    def clear_cache(self):
        with self._lock:
            self._tables.clear()

    def _table(self, luts_ptr, n_luts, device, cuda_stream):
        key = (device.index, luts_ptr, n_luts)
        with self._lock:
            t = self._tables.get(key)
            if t is not None:
                self._tables.move_to_end(key)
                return t
        t = torch.empty(_lib.TABLE_BYTES // 4, dtype=torch.int32, device=device)
        _lib.check(_lib.lib().ecf8_build_table(luts_ptr, n_luts, t.data_ptr(), cuda_stream), "_decode table")
        with self._lock:
            self._tables[key] = t
            while len(self._tables) > self.cache_size:
                self._tables.popitem(last=False)
        return t

    def __call__(self, grid, block, args, shared_mem=0, stream=None):
        if len(args) != 9:
            raise TypeError("args must be [luts, encoded, packed, output_positions, gaps, outputs, "
                            "n_luts, n_bytes, n_elements]")
        ptrs = [a.data_ptr() if isinstance(a, torch.Tensor) else int(a) for a in args[:6]]
        n_luts, n_bytes, n_elements = (int(a) for a in args[6:])
        tpb = int(block[0] if isinstance(block, (tuple, list)) else block)
        g = int(grid[0] if isinstance(grid, (tuple, list)) else grid)
        want = math.ceil(n_bytes / (tpb * self.bytes_per_thread))
        if g != want:
            raise ValueError(f"grid {g} does not cover {n_bytes} bytes (expected {want})")
        device = torch.device("cuda", torch.cuda.current_device())
        if stream is None:
            stream = torch.cuda.current_stream(device)
        cuda_stream = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream or 0)
        table = None
        if 2 <= n_luts <= _lib.MAX_LUTS and ptrs[0] and n_elements > 0:
            table = self._table(ptrs[0], n_luts, device, cuda_stream)
        arr = (_lib.Ecf8Stream * 1)(_lib.Ecf8Stream(
            ptrs[0], n_luts, 0, ptrs[1], n_bytes, ptrs[2], ptrs[3], max(g, 1), ptrs[4], g * tpb // 2, ptrs[5],
            n_elements, table.data_ptr() if table is not None else None))
        st = _lib.lib().ecf8_decode_batch(arr, 1, tpb, self.bytes_per_thread, cuda_stream)
        _lib.check(st, "_decode")


_decode = _DecodeLauncher()


# ---------------------------------------------------------------------------
# Hook
# ---------------------------------------------------------------------------

def _is_linear_like(m):
    return isinstance(m, nn.Linear) or (hasattr(m, "out_features") and hasattr(m, "in_features"))


def inject_weights(module, reconstructed):
    """Points the block's weight(s) at views of the decoded buffer
    (run.py:121-153)."""
    if isinstance(module, nn.Linear):
        module.weight = reconstructed.view(module.out_features, module.in_features)
    elif isinstance(module, nn.Embedding):
        module.weight = reconstructed.view(module.num_embeddings, module.embedding_dim)
    else:
        weights = torch.tensor_split(reconstructed, module.split_positions)
        for sub, w in zip(module.weight_injection_modules, weights):
            if _is_linear_like(sub):
                sub.weight = w.view(sub.out_features, sub.in_features)
            elif isinstance(sub, nn.Embedding):
                sub.weight = w.view(sub.num_embeddings, sub.embedding_dim)
            else:
                raise ValueError(f"Unsupported module type: {type(sub)}")


def _block_table(module):
    """The block's prepared decode table, built on first use on the current
    stream and kept as a non-persistent buffer (not part of the checkpoint).
    Returns (table, built now)."""
    device = module.encoded.device
    table = getattr(module, "ecf8_decode_table", None)
    if table is not None and table.device == device:
        return table, False
    table = build_decode_table(module.luts)
    module.register_buffer("ecf8_decode_table", table, persistent=False)
    return table, True


class _Prefetch:
    """Per-device state of the prefetching hook: a side stream, two scratch
    buffers (each the size of the largest block, allocated once, so no buffer
    is freed while a side-stream decode writes it) used in turn by
    consecutive blocks, the decodes in flight (block -> buffer index) and the
    events that order the two streams: per buffer, one recorded after the
    side-stream decode into it; one recorded on the compute stream before
    each side-stream decode.  An event is re-recorded only after every wait
    on its previous record has been enqueued."""

    def __init__(self, device, n_max):
        self.device = device
        self.side = torch.cuda.Stream(device)
        self.bufs = [torch.empty(n_max, dtype=torch.float8_e4m3fn, device=device) for _ in range(2)]
        self.pending = {}
        self.ready = [torch.cuda.Event(), torch.cuda.Event()]
        self.done = torch.cuda.Event()

    def buffer(self, i, n):
        return self.bufs[i][:n]


_PREFETCH = {}


def _n_elements(module):
    return module.packed_other_4bits.numel() * 2


def _decode_block(module, out, tpb, bpt, stream=None):
    table, fresh = _block_table(module)
    # The block's buffers and an existing table are written only at load
    # time, so the decode may start while the previous kernel on the stream
    # runs (it overwrites the scratch only after that kernel); right after
    # building the table it may not.
    decode_stream(module.luts, module.encoded, module.packed_other_4bits, module.output_positions,
                  module.gaps, out, tpb, bpt, table=table, overlap_previous=not fresh, stream=stream)


def get_hook(threads_per_block, bytes_per_thread):
    """forward_pre_hook that decodes a block's ECF8 stream into the device's
    shared scratch and injects the weight views (run.py:84-155).  With
    enable_decode_prefetch() on the model, the block's weights were decoded
    ahead on a side stream and the hook also starts the next block's decode."""

    def decode_hook(module, _):
        nxt = getattr(module, "_ecf8_next", None)
        if nxt is not None:
            _prefetch_hook(module, nxt, threads_per_block, bytes_per_thread)
            return
        device = module.encoded.device
        reconstructed = TensorManager.get_tensor(device, _n_elements(module))
        table, fresh = _block_table(module)
        key = (reconstructed.data_ptr(), table.data_ptr()) + tuple(module._buffers[k].data_ptr() for k in STREAM_BUFFERS)
        cached = module.__dict__.get("_ecf8_launch")
        if fresh or cached is None or cached[0] != key:
            # First decode of this block (or its buffers or the scratch moved):
            # checked launch, views injected, launch descriptor kept.
            _decode_block(module, reconstructed, threads_per_block, bytes_per_thread)
            inject_weights(module, reconstructed)
            s = {k: module._buffers[k] for k in STREAM_BUFFERS}
            module.__dict__["_ecf8_launch"] = (key, (_lib.Ecf8Stream * 1)(_stream_struct(s, reconstructed, table)))
            return
        # Later decodes: the same launch from the kept descriptor; the injected
        # views already point at this scratch.
        st = _lib.lib().ecf8_decode_batch_flags(cached[1], 1, threads_per_block, bytes_per_thread,
                                                _lib.DECODE_OVERLAP_PREVIOUS,
                                                torch.cuda.current_stream(device).cuda_stream)
        _lib.check(st, "ecf8_decode_batch_flags")

    return decode_hook


def _prefetch_launch(st, nxt, slot, tpb, bpt, ctas):
    """Side-stream decode of block `nxt` into buffer `slot`, from a launch
    descriptor checked and built once per (block, buffer)."""
    n = _n_elements(nxt)
    buf = st.buffer(slot, n)
    table = nxt.ecf8_decode_table
    key = (buf.data_ptr(), table.data_ptr()) + tuple(nxt._buffers[k].data_ptr() for k in STREAM_BUFFERS)
    kept = nxt.__dict__.setdefault("_ecf8_pf_launch", {})
    ent = kept.get(slot)
    if ent is None or ent[0] != key:
        s = {k: nxt._buffers[k] for k in STREAM_BUFFERS}
        _check_stream(s, buf, st.device, table)
        ent = kept[slot] = (key, (_lib.Ecf8Stream * 1)(_stream_struct(s, buf, table)))
    rc = _lib.lib().ecf8_decode_batch_flags(ent[1], 1, tpb, bpt, _lib.decode_ctas(ctas) if ctas else 0,
                                            st.side.cuda_stream)
    _lib.check(rc, "ecf8_decode_batch_flags")


def _prefetch_hook(module, nxt, tpb, bpt):
    device = module.encoded.device
    st = _PREFETCH.get(device)
    if st is None or st.bufs[0].numel() < max(_n_elements(module), _n_elements(nxt)):
        n_max = max([_n_elements(m) for m in _prefetch_blocks(module)] + [_n_elements(module), _n_elements(nxt)])
        st = _PREFETCH[device] = _Prefetch(device, n_max)
    cur = torch.cuda.current_stream(device)
    slot = st.pending.pop(module, None)
    if slot is not None:  # decoded ahead: wait for that decode on this stream
        cur.wait_event(st.ready[slot])
    else:  # not decoded ahead (first block of a forward, or another order): decode here,
        # after every side-stream decode still writing either buffer
        cur.wait_stream(st.side)
        slot = 0 if 0 not in st.pending.values() else 1
        st.pending = {m: v for m, v in st.pending.items() if v != slot}
        _decode_block(module, st.buffer(slot, _n_elements(module)), tpb, bpt)
    # Views: injected when the block's weights do not already view this buffer.
    views = (slot, st.bufs[slot].data_ptr())
    if module.__dict__.get("_ecf8_pf_views") != views:
        inject_weights(module, st.buffer(slot, _n_elements(module)))
        module.__dict__["_ecf8_pf_views"] = views
    # The next block goes into the other buffer once everything enqueued so far
    # on this stream is done (that buffer was read by the block before this one).
    other = 1 - slot
    st.pending = {m: v for m, v in st.pending.items() if v != other}
    _block_table(nxt)  # built on this stream at first use, before the side stream waits for it
    st.done.record(cur)
    st.side.wait_event(st.done)
    _prefetch_launch(st, nxt, other, tpb, bpt, module.__dict__.get("_ecf8_prefetch_ctas", 0))
    st.ready[other].record(st.side)
    st.pending[nxt] = other


def _prefetch_blocks(module):
    return getattr(module, "_ecf8_blocks", None) or [module]


def enable_decode_prefetch(model, enable=True, ctas=0):
    """Decode-ahead mode of the forward-pre-hook: each hooked block, in module
    order (the forward order of decoder layers and DiT blocks), starts the
    next block's decode on a side stream into the second of two per-device
    scratch buffers, and its own hook only waits for the decode started one
    block earlier.  The decode can then run while the GPU would otherwise wait
    for the host to launch the current block's kernels; decoded bytes, and so
    outputs, are the same as with the plain hook.  It pays only where the
    forward leaves the GPU idle between launches: a decode holds every SM
    while it runs, so it does not share them with the block's own kernels,
    and the mode costs some host time per block (the batch-16 Qwen3-8B
    generation of the benchmark, whose step keeps the GPU busy, runs slower
    with it: 0.918 against 0.948 of the uncompressed tokens/s).  `ctas` > 0
    limits the side-stream decodes to that many CTAs (of one per SM), so they
    take only part of the GPU and the block's own kernels keep the rest (on
    that generation: 0.913 with 32 CTAs, 0.904 with 74).  Uses
    two scratch buffers of the largest block instead of one.  The last block
    prefetches the first (the next forward).  Returns the number of hooked
    blocks.  enable=False restores the plain hook."""
    blocks = [m for m in model.modules() if "encoded" in m._buffers and "luts" in m._buffers
              and any(getattr(h, "__name__", "") == "decode_hook" for h in m._forward_pre_hooks.values())]
    for i, m in enumerate(blocks):
        # plain attributes: assigning a module through nn.Module would make it a child
        object.__setattr__(m, "_ecf8_next", blocks[(i + 1) % len(blocks)] if enable else None)
        object.__setattr__(m, "_ecf8_blocks", blocks if enable else None)
        object.__setattr__(m, "_ecf8_prefetch_ctas", int(ctas) if enable else 0)
        # Either hook's kept launch state assumes the weights view its own
        # buffers: switching modes re-injects the views on the next decode.
        for k in ("_ecf8_launch", "_ecf8_pf_views", "_ecf8_pf_launch"):
            m.__dict__.pop(k, None)
    if not enable:
        _PREFETCH.clear()
    return len(blocks)


# ---------------------------------------------------------------------------
# Loaders
# ---------------------------------------------------------------------------

def _shared_mem_size(module, threads_per_block):
    op = module.output_positions.view(torch.uint64).to(torch.int64)
    per_group = (op[1:] - op[:-1]).max().item() if op.numel() > 1 else 0
    return threads_per_block * 4 + 4 + int(per_group)


def _process_compressed_tensor(module, attr_name, tensor_value, tensor_name, pattern_dict,
                               threads_per_block, bytes_per_thread):
    """Registers one ECF8 buffer on its block; on `encoded` adds the hook and
    removes the dense weights, on `output_positions` records the reference's
    shared-memory size (run.py:406-458)."""
    if attr_name == "split_positions":
        module.split_positions = tensor_value.tolist()
    else:
        module.register_buffer(attr_name, tensor_value)
    if attr_name == "encoded":
        module.register_forward_pre_hook(get_hook(threads_per_block, bytes_per_thread))
        module_path = ".".join(tensor_name.split(".")[:-1])
        for pattern, attr_names in pattern_dict.items():
            if re.fullmatch(pattern, module_path):
                if isinstance(module, (nn.Embedding, nn.Linear)):
                    if "weight" in module._parameters or hasattr(module, "weight"):
                        delattr(module, "weight")
                else:
                    module.weight_injection_modules = []
                    for attr_path in attr_names:
                        target = module
                        for p in attr_path.split("."):
                            target = getattr(target, p)
                        if not hasattr(target, "weight"):
                            raise ValueError(f"Weight not found for {attr_path}")
                        delattr(target, "weight")
                        module.weight_injection_modules.append(target)
                break
    elif attr_name == "output_positions":
        module.shared_mem_size = _shared_mem_size(module, threads_per_block)


def _module_at(model, tensor_name):
    module = model
    for part in tensor_name.split(".")[:-1]:
        if not hasattr(module, part):
            print(f"Cannot find module path for {tensor_name}", file=stderr)
            return None
        module = getattr(module, part)
    return module


def _load_one(model, tensor_name, tensor_value, params, buffers, state_keys, pattern_dict, tpb, bpt):
    from .fp8_model import fused_experts_owner
    fused = fused_experts_owner(model, tensor_name)
    if fused is not None:  # one expert's tensor of a fused expert block (per-expert checkpoint keys)
        owner, m, key = fused
        owner.load_expert_tensor(m, key, tensor_value, tpb, bpt)
        return
    if tensor_name in state_keys:
        target = params.get(tensor_name)
        if target is None:
            target = buffers[tensor_name]
        if target.shape == tensor_value.shape:
            target.data = tensor_value
        else:
            print(f"Shape mismatch for {tensor_name}: model {target.shape} vs loaded "
                  f"{tensor_value.shape}", file=stderr)
        return
    module = _module_at(model, tensor_name)
    if module is not None:
        _process_compressed_tensor(module, tensor_name.split(".")[-1], tensor_value, tensor_name,
                                   pattern_dict, tpb, bpt)


def load_and_replace_tensors(model, directory_path, dfloat_config):
    """Loads every .safetensors file of a compressed checkpoint into `model`
    (run.py:158-275): known parameters/buffers are replaced, ECF8 buffers are
    registered on their blocks together with the decode hook."""
    from safetensors.torch import load_file
    tpb = dfloat_config["threads_per_block"]
    bpt = dfloat_config["bytes_per_thread"]
    pattern_dict = dfloat_config["pattern_dict"]["fp8"]
    files = sorted(f for f in os.listdir(directory_path) if f.endswith(".safetensors"))
    for name in files:
        tensors = load_file(os.path.join(directory_path, name))
        params = dict(model.named_parameters())
        buffers = dict(model.named_buffers())
        keys = set(model.state_dict().keys())
        for tname, tval in tensors.items():
            _load_one(model, tname, tval, params, buffers, keys, pattern_dict, tpb, bpt)
    return model


def load_and_replace_tensors_parallel(model, directory_path, dfloat_config):
    """As load_and_replace_tensors, reading files on a thread pool (run.py:278-403)."""
    from concurrent.futures import ThreadPoolExecutor
    from safetensors.torch import load_file
    tpb = dfloat_config["threads_per_block"]
    bpt = dfloat_config["bytes_per_thread"]
    pattern_dict = dfloat_config["pattern_dict"]["fp8"]
    params = dict(model.named_parameters())
    buffers = dict(model.named_buffers())
    keys = set(model.state_dict().keys())
    files = sorted(f for f in os.listdir(directory_path) if f.endswith(".safetensors"))
    workers = min(4 if len(files) > 20 else 8, max(len(files), 1), os.cpu_count() or 4)
    lock = threading.Lock()

    def work(name):
        try:
            tensors = load_file(os.path.join(directory_path, name))
        except Exception as e:  # same policy as the reference: report and go on
            print(f"Error loading {name}: {e}", file=stderr)
            return 0
        with lock:  # module registration mutates the model
            for tname, tval in tensors.items():
                _load_one(model, tname, tval, params, buffers, keys, pattern_dict, tpb, bpt)
        return len(tensors)

    with ThreadPoolExecutor(max_workers=workers) as ex:
        total = sum(ex.map(work, files))
    print(f"Processed {total} tensors from {len(files)} files", file=stderr)
    return model


def get_dfloat_model_name_or_path(repo_id: str, dfloat_dir: str = "../dfloat-models"):
    """(local directory, hub id) of the compressed checkpoint of `repo_id`
    (run.py:473-480)."""
    parts = repo_id.split("/")
    parts[0] = "DFloat11"
    return (os.path.join(dfloat_dir, "models--" + "--".join(parts) + "-DF6.5"),
            "/".join(parts) + "-DF6.5")


def param_to_bytes(param):
    return param.numel() * param.element_size()


def report_model_size(model, include_pattern):
    """(included GB, excluded GB, total GB) of a model's state (dfloat/utils.py:24-67)."""
    inc = exc = 0
    for name, p in model.state_dict().items():
        if include_pattern is None:
            hit = True
        elif isinstance(include_pattern, dict):
            hit = any(re.search(pat, name) and any(a in name or name.endswith(a) for a in attrs)
                      for pat, attrs in include_pattern.items())
        else:
            hit = any(re.search(pat, name) for pat in include_pattern)
        if hit:
            inc += param_to_bytes(p)
        else:
            exc += param_to_bytes(p)
    gb = 1024 ** 3
    return inc / gb, exc / gb, (inc + exc) / gb


def get_no_split_classes(model, patterns):
    """Class names of the modules whose full name matches one of `patterns`
    (run.py:461-470): the blocks accelerate must not split across devices."""
    out = []
    for name, m in model.named_modules():
        if any(re.fullmatch(p, name) for p in patterns):
            if m.__class__.__name__ not in out:
                out.append(m.__class__.__name__)
    return out


def _is_fp8_config(path):
    try:
        with open(os.path.join(path, "config.json")) as f:
            q = json.load(f).get("quantization_config") or {}
    except OSError:
        return False
    return q.get("quant_method") == "fp8"


def _load_original_model(dfloat_repo_id, model_name_or_path, trust_remote_code=True, **kwargs):
    """The model the compressed blocks go into.  An FP8 checkpoint (config.json
    with an fp8 quantization_config) is assembled by ecf8_b200.fp8_model, since
    transformers needs accelerate and hub kernels for it: from the original
    directory when it is on disk, else from the compressed checkpoint's own
    config (its safetensors then supply every tensor).  Other models load
    through transformers as in run.py:483-500."""
    from .fp8_model import fp8_model_from_config, load_fp8_checkpoint
    dtype = kwargs.get("torch_dtype", kwargs.get("dtype", torch.bfloat16))
    if os.path.isdir(model_name_or_path) and _is_fp8_config(model_name_or_path):
        return load_fp8_checkpoint(model_name_or_path, device="cpu", dtype=dtype)
    if _is_fp8_config(dfloat_repo_id):
        from transformers import AutoConfig
        return fp8_model_from_config(AutoConfig.from_pretrained(dfloat_repo_id), device="cpu", seed=None,
                                     dtype=dtype)
    from transformers import AutoModelForCausalLM
    return AutoModelForCausalLM.from_pretrained(
        model_name_or_path, trust_remote_code=trust_remote_code, dtype=dtype,
        attn_implementation=kwargs.get("attn_implementation"), low_cpu_mem_usage=True)


class DFloatModel:
    @classmethod
    def from_pretrained(cls, dfloat_repo_id: str, dfloat_model_id: str, model_name_or_path: str,
                        device: Optional[str] = None, device_map: str = "auto",
                        max_memory: Optional[Dict[Union[int, str], Union[int, str]]] = None,
                        trust_remote_code: bool = True, **kwargs):
        """Loads the original FP8 model, swaps its FP8 blocks for ECF8 streams
        decoded on the fly, and places it (run.py:483-566).  The checkpoint
        must already be on disk (this build has no network); device_map="auto"
        places the whole model on the current GPU when accelerate is absent."""
        if not os.path.exists(dfloat_repo_id):
            raise FileNotFoundError(
                f"{dfloat_repo_id} not found (download of {dfloat_model_id} is not available here)")
        from transformers import AutoConfig
        model = _load_original_model(dfloat_repo_id, model_name_or_path, trust_remote_code, **kwargs)
        model.eval()
        config = AutoConfig.from_pretrained(dfloat_repo_id)
        assert hasattr(config, "dfloat_config")
        dfloat_config = dict(config.dfloat_config)
        with open(os.path.join(dfloat_repo_id, "pattern_dict.json")) as f:
            dfloat_config["pattern_dict"] = json.load(f)
        fp8_patterns = dfloat_config["pattern_dict"]["fp8"]
        inc, exc, tot = report_model_size(model, fp8_patterns)
        with open(os.path.join(dfloat_repo_id, "model_size.csv"), "w") as f:
            f.write("fp8_blocks,rest,total\n")
            f.write(f"{inc},{exc},{tot}\n")
        load_and_replace_tensors_parallel(model, dfloat_repo_id, dfloat_config)
        _, _, tot = report_model_size(model, None)
        with open(os.path.join(dfloat_repo_id, "model_size.csv"), "a") as f:
            f.write(f"{tot - exc},{exc},{tot}\n")
        if device:
            model = model.to(device)
        else:
            assert device_map == "auto", 'device_map should be "auto" if no specific device is provided.'
            try:
                from accelerate import dispatch_model, infer_auto_device_map
                from accelerate.utils import get_balanced_memory
            except ImportError:
                model = model.to(torch.device("cuda", torch.cuda.current_device()))
            else:
                classes = get_no_split_classes(model, get_default_no_split_pattern(model.__class__.__name__))
                mm = get_balanced_memory(model, max_memory=max_memory, no_split_module_classes=classes)
                dm = infer_auto_device_map(model, max_memory=mm, no_split_module_classes=classes)
                model = dispatch_model(model, dm)
        if any(p.device.type == "cpu" for p in model.parameters()):
            print("Warning: Some model layers are on CPU.", file=stderr)
        return model


class DFloatDiffSynthModelFP8:
    @classmethod
    def from_pretrained(cls, dfloat_repo_id: str, dfloat_model_id: str, model_name_or_path: str,
                        device: Optional[str] = "cuda"):
        """DiffSynth pipelines with ECF8 blocks (run.py:569-729).  Needs the
        `diffsynth` package, which this environment does not have."""
        try:
            import diffsynth  # noqa: F401
        except ImportError as e:
            raise ImportError("DFloatDiffSynthModelFP8 needs the diffsynth package") from e
        raise NotImplementedError("DiffSynth pipelines are not wired up in this build")


# ---------------------------------------------------------------------------
# Host-buffer decode (streams and outputs in host memory)
# ---------------------------------------------------------------------------

class HostStreamDecoder:
    """Decodes ECF8 streams whose buffers live in host memory into host
    outputs, e.g. to decompress a checkpoint held in RAM.  Each stream is
    copied in, decoded and copied out through one of `depth` device staging
    slots; copies in, decodes and copies out of consecutive streams overlap
    on three CUDA streams.  Host tensors should be pinned for the copies to
    be asynchronous.  Staging buffers are allocated once, for the largest
    stream seen, and reused."""

    def __init__(self, device=None, depth=2):
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.depth = depth
        self.slots = [None] * depth
        self.cap = {}
        with torch.cuda.device(self.device):
            self.s_in = torch.cuda.Stream(self.device)
            self.s_dec = torch.cuda.Stream(self.device)
            self.s_out = torch.cuda.Stream(self.device)
        self.free = [None] * depth  # event: slot may be overwritten

    def _slot(self, i, s):
        need = {k: s[k].numel() * s[k].element_size() for k in STREAM_BUFFERS}
        need["out"] = s["packed_other_4bits"].numel() * 2
        slot = self.slots[i]
        if slot is None or any(slot[k].numel() < need[k] for k in need):
            slot = {k: torch.empty(max(need[k], 16), dtype=torch.uint8, device=self.device) for k in need}
            self.slots[i] = slot
        return slot, need

    def decode(self, streams, outs, tables=None):
        """streams: list of dicts with the five buffers (host tensors);
        outs: matching host uint8/e4m3 tensors; tables: optional prepared
        decode tables (device tensors, build_decode_table).  Returns when all
        are done."""
        for j, (s, o) in enumerate(zip(streams, outs)):
            i = j % self.depth
            slot, need = self._slot(i, s)
            with torch.cuda.stream(self.s_in):
                if self.free[i] is not None:
                    self.s_in.wait_event(self.free[i])
                views = {}
                for k in STREAM_BUFFERS:
                    src = s[k].reshape(-1).view(torch.uint8)
                    dst = slot[k][:need[k]]
                    dst.copy_(src, non_blocking=True)
                    views[k] = dst
                ev_in = torch.cuda.Event()
                ev_in.record(self.s_in)
            self.s_dec.wait_event(ev_in)
            n = need["out"]
            out_dev = slot["out"][:n]
            decode_stream(views["luts"].view(s["luts"].shape), views["encoded"], views["packed_other_4bits"],
                          views["output_positions"], views["gaps"], out_dev, stream=self.s_dec,
                          table=tables[j] if tables is not None else None)
            ev_dec = torch.cuda.Event()
            ev_dec.record(self.s_dec)
            self.s_out.wait_event(ev_dec)
            with torch.cuda.stream(self.s_out):
                o.reshape(-1).view(torch.uint8)[:n].copy_(out_dev, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.s_out)
            self.free[i] = ev
        self.s_out.synchronize()
        return outs
