"""ECF8 compressor: an FP8 checkpoint -> a compressed checkpoint in the
reference's on-disk layout (zeyuyang8/ecf8 scripts/compress.py).

    python -m ecf8_b200.compress --repo_id <FP8 checkpoint dir> --save_model --validate_cuda

Per block matched by the model family's FP8 pattern (`get_fp8_pattern_dict`,
dfloat/const.py) the block's e4m3 Linear weights are flattened in sorted name
order, split into exponents and sign+mantissa nibbles, Huffman coded (codes of
at most 16 bits plus EOF) and packed into the five stream buffers.  The
reference does this on CPU worker processes with a Python packer (about a
minute per 8B layer); here the packer runs on the GPU (ecf8_encode_plan /
ecf8_encode_emit), one block after another.

Output, as the reference writes it (compress.py:239-247, 587-680):
  <save_path>/cache/<block>.safetensors   flat_weights, luts, encoded,
                                          packed_other_4bits, output_positions
                                          (u64 as bytes), gaps, split_positions
  <save_path>/cache/<block>.pkl           block metadata
  <save_path>/entropy.csv                 exponent entropy per block
  <save_path>/pattern_dict.json           {"fp8": {regex: [layer names]}, "bf16": {...}}
  <save_path>/config.json, *.safetensors  with --save_model: the model with its
                                          FP8 blocks replaced by the buffers and
                                          config.dfloat_config
<save_path> is get_dfloat_model_name_or_path(repo_id, dfloat_dir)[0].
"""

import argparse
import json
import operator
import os
import pickle
import re
import shutil
import sys
import time

import torch
import torch.nn as nn

from .codec import (
    compress_fp8,
    find_layers_by_data_type_and_layer_type,
    find_layers_by_selection,
    flatten_block_of_weights,
    locate_block_by_regex,
)
from .const import get_fp8_pattern_dict
from .fp8_model import Fp8FusedExperts, Fp8Linear, fused_experts_owner, load_fp8_checkpoint
from .run import decode_stream, get_dfloat_model_name_or_path

package_version = "0.2.0"

STREAM_KEYS = ("luts", "encoded", "packed_other_4bits", "output_positions", "gaps", "split_positions")


def _fp8_layer_types():
    types = [nn.Linear, Fp8Linear]
    try:
        from transformers.integrations.finegrained_fp8 import FP8Linear
        types.append(FP8Linear)
    except Exception:
        pass
    return types


def validate_cuda_decoding_fp8(result, tensors, device):
    """Decodes a block's stream on `device` and checks it against the
    block's flat weights (compress.py:70-127)."""
    dev = torch.device(device)
    out = torch.empty(tensors["packed_other_4bits"].numel() * 2, dtype=torch.uint8, device=dev)
    decode_stream(tensors["luts"].to(dev), tensors["encoded"].to(dev), tensors["packed_other_4bits"].to(dev),
                  tensors["output_positions"].to(dev), tensors["gaps"].to(dev), out,
                  result["threads_per_block"], result["bytes_per_thread"])
    torch.cuda.synchronize(dev)
    if not torch.equal(out.cpu(), tensors["flat_weights"].view(torch.uint8).cpu()):
        raise AssertionError(f"CUDA decode of {result['block_name']} differs from its weights")


def _block_tensors(layers, device):
    flat, split_positions = flatten_block_of_weights(layers, dtype=torch.float8_e4m3fn)
    c = compress_fp8(flat, device=device)
    tensors = {
        "flat_weights": flat,
        "luts": c["luts"].cpu(),
        "encoded": c["encoded"].cpu(),
        "packed_other_4bits": c["packed_other_4bits"].cpu(),
        "output_positions": c["output_positions"].view(torch.uint8).cpu(),
        "gaps": c["gaps"].cpu(),
        "split_positions": split_positions,
    }
    return tensors, c["entropy"]


def _entropy_of(flat):
    from .codec import compute_shannon_entropy, get_exponents_and_other_4bits_fp8_e4m3
    exps, _ = get_exponents_and_other_4bits_fp8_e4m3(flat.reshape(-1))
    return compute_shannon_entropy(exps)


def process_fp8_block(block_item, info_dict, print_time=False):
    """Compresses one block into cache/<block>.safetensors and returns its
    metadata (compress.py:130-270).  A block already in the cache is reused."""
    from safetensors.torch import load_file, save_file
    block_name, layers = block_item
    save_path = info_dict["save_path"]
    cache_dir = os.path.join(save_path, "cache")
    os.makedirs(cache_dir, exist_ok=True)
    block_save_path = os.path.join(cache_dir, block_name + ".safetensors")
    metadata_save_path = os.path.join(cache_dir, block_name + ".pkl")

    layer_names, layers_to_delete = [], []
    for full in layers:
        if not (full.startswith(block_name + ".") or full == block_name):
            raise ValueError(f"layer name {full} is not inside block {block_name}")
        layers_to_delete.append(full)
        layer_names.append(full[len(block_name) + 1:])
    matched_regex = next((r for r in info_dict["model_fp8_regex"] if re.fullmatch(r, block_name)), None)

    entropy = None
    if os.path.exists(block_save_path):
        if os.path.exists(metadata_save_path):
            with open(metadata_save_path, "rb") as f:
                entropy = pickle.load(f).get("entropy")
        if entropy is None:
            entropy = _entropy_of(load_file(block_save_path)["flat_weights"])
    else:
        t0 = time.time()
        tensors, entropy = _block_tensors(layers, info_dict.get("device"))
        save_file(tensors, block_save_path)
        if print_time:
            print(f"{block_name}: compressed in {time.time() - t0:.2f}s", file=sys.stderr)

    metadata = {
        "block_name": block_name,
        "layer_names": layer_names,
        "matched_regex": matched_regex,
        "layers_to_delete": layers_to_delete,
        "threads_per_block": info_dict["threads_per_block"],
        "bytes_per_thread": info_dict["bytes_per_thread"],
        "block_save_path": block_save_path,
        "entropy": entropy,
    }
    with open(metadata_save_path, "wb") as f:
        pickle.dump(metadata, f)
    return metadata


def process_all_fp8_blocks_parallel(fp8_layers_by_block, num_processes=1, reverse=False, info_dict=None):
    """All blocks, in name order (reversed with `reverse`), as compress.py:303-341
    does with a process pool; the GPU packer makes a pool unnecessary, so
    `num_processes` is accepted for the same call and not used."""
    items = sorted(fp8_layers_by_block.items(), reverse=reverse)
    return [process_fp8_block(item, info_dict) for item in items]


def find_fp8_blocks(model, model_fp8_regex):
    """{block name: {layer name: module}} for a family's FP8 pattern: a list of
    block regexes (every e4m3 Linear inside), or {regex: [layer paths]}
    (compress.py:506-537).  Experts held in a fused block (Fp8FusedExperts,
    transformers' 3-D expert parameters) count as the per-expert blocks
    "<experts>.M" of the reference layout, with views as their sub-Linears."""
    blocks = {}
    if isinstance(model_fp8_regex, list):
        joined = "|".join(model_fp8_regex)
        for block_name, block in locate_block_by_regex(model, joined).items():
            blocks[block_name] = find_layers_by_data_type_and_layer_type(
                block, target_dtype=torch.float8_e4m3fn, layers=_fp8_layer_types(), name=block_name)
        for name, mod in model.named_modules():
            if isinstance(mod, Fp8FusedExperts) and mod._has_dense():
                for m in range(mod.num_experts):
                    if re.fullmatch(joined, f"{name}.{m}"):
                        blocks[f"{name}.{m}"] = mod.expert_layers(m, f"{name}.{m}")
    else:
        for regex, selected in model_fp8_regex.items():
            for block_name, block in locate_block_by_regex(model, regex).items():
                blocks[block_name] = find_layers_by_selection(block, selected, name=block_name)
    return {k: v for k, v in blocks.items() if v}


def _delete_layer_weights(model, block_name, sub_module, layers_to_delete):
    """Drops the compressed layers' dense weights.  The reference drops the
    whole sub-Linear modules (compress.py:583-600) and takes their scales from
    the original checkpoint at load time; keeping the modules keeps
    `weight_scale_inv` in the compressed checkpoint, so it loads on its own
    (and the reference loader, which overwrites known keys, reads it too)."""
    for layer_name in layers_to_delete:
        layer = sub_module if layer_name == block_name else operator.attrgetter(layer_name)(model)
        if not isinstance(layer, (nn.Linear, nn.Embedding, Fp8Linear)) and not hasattr(layer, "weight"):
            raise ValueError(f"Unsupported layer type {type(layer)}")
        delattr(layer, "weight")


def compress_model(model, save_path, threads_per_block=512, bytes_per_thread=8, validate_cuda=False,
                   save_model=False, tokenizer_path=None, device=None, reverse=False, print_time=False):
    """Compresses every FP8 block of `model` into `save_path`, replaces the
    blocks' weights by the stream buffers, and (save_model) writes the
    compressed checkpoint.  Returns the pattern dict (compress.py:495-680)."""
    from safetensors.torch import load_file, save_file
    device = device or ("cuda" if torch.cuda.is_available() else None)
    if device is None:
        raise RuntimeError("the ECF8 packer runs on a CUDA device")
    os.makedirs(save_path, exist_ok=True)
    pattern = get_fp8_pattern_dict(model.__class__.__name__)
    model_fp8_regex = pattern["fp8"]
    fp8_regex_dict = {r: None for r in model_fp8_regex}
    bf16_regex_dict = {r: [] for r in pattern["bf16"]}
    info_dict = {"save_path": save_path, "model_fp8_regex": list(model_fp8_regex),
                 "bytes_per_thread": bytes_per_thread, "threads_per_block": threads_per_block,
                 "device": device}
    blocks = find_fp8_blocks(model, model_fp8_regex)
    results = [process_fp8_block(item, info_dict, print_time)
               for item in sorted(blocks.items(), reverse=reverse)]

    entropy_rows = {}
    for result in results:
        block_name = result["block_name"]
        entropy_rows[block_name] = result["entropy"]
        tensors = load_file(result["block_save_path"])
        if validate_cuda:
            validate_cuda_decoding_fp8(result, tensors, device)
        fused = fused_experts_owner(model, block_name + ".encoded")
        if fused is not None:  # one expert of a fused block: the block drops its dense weights itself
            owner, m, _ = fused
            for key in STREAM_KEYS:
                owner.add_expert_stream(m, key, tensors[key], threads_per_block, bytes_per_thread)
        else:
            sub_module = operator.attrgetter(block_name)(model)
            _delete_layer_weights(model, block_name, sub_module, result["layers_to_delete"])
            for key in STREAM_KEYS:
                sub_module.register_buffer(key, tensors[key])
        matched = result["matched_regex"]
        if matched:
            if fp8_regex_dict[matched] is None:
                fp8_regex_dict[matched] = result["layer_names"]
            elif fp8_regex_dict[matched] != result["layer_names"]:
                raise ValueError(f"block {block_name} has layers {result['layer_names']}, other blocks of "
                                 f"{matched} have {fp8_regex_dict[matched]}")

    with open(os.path.join(save_path, "entropy.csv"), "w") as f:
        f.write("block_name,entropy\n")
        for name in sorted(entropy_rows):
            f.write(f"{name},{entropy_rows[name]}\n")
    regex_json = {"fp8": fp8_regex_dict, "bf16": bf16_regex_dict}

    if save_model:
        dfloat_config = {"version": package_version, "threads_per_block": threads_per_block,
                         "bytes_per_thread": bytes_per_thread}
        cfg = model.config.to_dict()
        cfg["dfloat_config"] = dfloat_config
        with open(os.path.join(save_path, "config.json"), "w") as f:
            json.dump(cfg, f, indent=2)
        state = {k: v.detach().contiguous().cpu() for k, v in model.state_dict().items()}
        if getattr(model.config, "tie_word_embeddings", False):
            state.pop("lm_head.weight", None)
        save_file(state, os.path.join(save_path, "model.safetensors"))
        if tokenizer_path:
            for name in os.listdir(tokenizer_path):
                if name.startswith("tokenizer") or name in ("special_tokens_map.json", "vocab.json", "merges.txt"):
                    shutil.copy(os.path.join(tokenizer_path, name), save_path)
    with open(os.path.join(save_path, "pattern_dict.json"), "w") as f:
        json.dump(regex_json, f, indent=4)
    return regex_json


def main(argv=None):
    ap = argparse.ArgumentParser(description="Compress an FP8 checkpoint into ECF8 streams.")
    ap.add_argument("--config", type=str, default=None, help="toml with [download] dfloat_dir")
    ap.add_argument("--repo_id", type=str, default="Qwen/Qwen3-8B-FP8",
                    help="local FP8 checkpoint directory (no hub download here)")
    ap.add_argument("--dfloat_dir", type=str, default=None)
    ap.add_argument("--bytes_per_thread", type=int, default=8)
    ap.add_argument("--threads_per_block", type=int, default=512)
    ap.add_argument("--save_model", action="store_true")
    ap.add_argument("--n_processes", type=int, default=36, help="accepted; the GPU packer needs no pool")
    ap.add_argument("--sequential", action="store_true")
    ap.add_argument("--reverse", action="store_true")
    ap.add_argument("--validate_cuda", action="store_true")
    ap.add_argument("--thread_pool", action="store_true")
    ap.add_argument("--model_name", type=str, default=None,
                    help="hub name the compressed directory is named after (default: --repo_id)")
    args = ap.parse_args(argv)
    dfloat_dir = args.dfloat_dir
    if dfloat_dir is None and args.config:
        import tomllib
        with open(args.config, "rb") as f:
            dfloat_dir = tomllib.load(f)["download"]["dfloat_dir"]
    dfloat_dir = dfloat_dir or "../dfloat-models"
    if not os.path.isdir(args.repo_id):
        raise SystemExit(f"{args.repo_id}: not a local checkpoint directory (no network here)")
    model = load_fp8_checkpoint(args.repo_id, device="cpu")
    name = args.model_name or args.repo_id.rstrip("/")
    save_path, _ = get_dfloat_model_name_or_path(name, dfloat_dir)
    regex_json = compress_model(model, save_path, args.threads_per_block, args.bytes_per_thread,
                                args.validate_cuda, args.save_model, tokenizer_path=args.repo_id,
                                reverse=args.reverse, print_time=True)
    print(json.dumps(regex_json))
    return save_path


if __name__ == "__main__":
    main()


def compress_model_in_place(model, threads_per_block=512, bytes_per_thread=8, device=None):
    """Compresses every FP8 block of a model already on the GPU and wires the
    decode-before-forward hook, without touching disk: the state a model has
    after compress + DFloatModel.from_pretrained.  Returns the pattern dict."""
    from .run import _process_compressed_tensor
    device = device or next(model.parameters()).device
    pattern = get_fp8_pattern_dict(model.__class__.__name__)
    blocks = find_fp8_blocks(model, pattern["fp8"])
    fp8_regex_dict = {}
    for block_name, layers in sorted(blocks.items()):
        names = [n[len(block_name) + 1:] for n in layers]
        regex = next(r for r in pattern["fp8"] if re.fullmatch(r, block_name))
        fp8_regex_dict.setdefault(regex, names)
        flat, split_positions = flatten_block_of_weights(layers, dtype=torch.float8_e4m3fn)
        c = compress_fp8(flat.to(device), device=device)
        del flat
        tensors = {"luts": c["luts"], "encoded": c["encoded"], "packed_other_4bits": c["packed_other_4bits"],
                   "output_positions": c["output_positions"].view(torch.uint8), "gaps": c["gaps"],
                   "split_positions": split_positions}
        fused = fused_experts_owner(model, block_name + ".encoded")
        if fused is not None:
            owner, m, _ = fused
            for key in ("luts", "packed_other_4bits", "output_positions", "gaps", "split_positions", "encoded"):
                owner.add_expert_stream(m, key, tensors[key], threads_per_block, bytes_per_thread)
            continue
        module = operator.attrgetter(block_name)(model)
        for key in ("luts", "packed_other_4bits", "output_positions", "gaps", "split_positions", "encoded"):
            _process_compressed_tensor(module, key, tensors[key], f"{block_name}.{key}", {regex: names},
                                       threads_per_block, bytes_per_thread)
    return {"fp8": fp8_regex_dict, "bf16": {r: [] for r in pattern["bf16"]}}
