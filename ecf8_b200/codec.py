"""ECF8 stream producers: exponent split, code table, LUTs and the GPU packer.

Same names, arguments and outputs as the reference codec in
zeyuyang8/ecf8 dfloat/utils.py, so a compressor written against it runs
unchanged:

  flatten_block_of_weights               utils.py:188-204
  get_exponents_and_other_4bits_fp8_e4m3 utils.py:207-227
  compute_shannon_entropy                utils.py:230-236
  get_nbit_codec                         utils.py:239-267
  get_luts_from_huffman_table            utils.py:270-370
  encode_exponents_for_cuda              utils.py:502-530 (packer 373-499)
  repo_id_to_model_id, locate_block_by_regex, find_layers_by_*
                                         utils.py:70-185

The LUT layout and the stream layout are the format contract and are
reproduced exactly.  The code table is this package's own: a Huffman code
(lengths from the usual two-smallest merge, ties broken by symbol) in
canonical order, with an EOF pseudo-symbol of frequency 1 as the reference's
dahuffman dependency adds.  It differs from dahuffman's tie-breaking, which
only changes which valid prefix code a block gets; any prefix code of at most
16 bits is a valid ECF8 stream for every decoder.  Canonical codes also give
every LUT row an entry at byte 0, so no bit pattern resolves to a length-0
code.

The packer runs on the GPU (ecf8_encode_plan / ecf8_encode_emit) and is
byte-identical to the reference packer for the same code table.
"""

import ctypes
import heapq
import math
import re

import numpy as np
import torch

from . import _lib

MAX_CODE_BITS = 16


class _EndOfFile:
    """The EOF pseudo-symbol of a code table (ordered after all real symbols)."""

    def __repr__(self):
        return "_EOF"

    def __hash__(self):
        return hash("ecf8-eof")

    def __eq__(self, other):
        return isinstance(other, _EndOfFile)

    def __lt__(self, other):
        return False

    def __gt__(self, other):
        return not isinstance(other, _EndOfFile)


EOF = _EndOfFile()


class HuffmanCode:
    """A code table with the attributes the reference codec reads from its
    dahuffman codec: ``_table`` (symbol -> (bit_count, value)), ``_eof`` and
    ``get_code_table()`` (utils.py:241,408,447)."""

    def __init__(self, table, eof=EOF):
        self._table = dict(table)
        self._eof = eof

    def get_code_table(self):
        return self._table

    @classmethod
    def from_frequencies(cls, frequencies):
        return cls(huffman_code_table(frequencies))


def huffman_code_lengths(frequencies):
    """{symbol: frequency} (EOF added with frequency 1) -> {symbol: length}."""
    freqs = dict(frequencies)
    if EOF not in freqs:
        freqs[EOF] = 1
    order = sorted(freqs, key=lambda s: (isinstance(s, _EndOfFile), s if isinstance(s, int) else 0))
    if len(order) == 1:
        return {order[0]: 1}
    # (frequency, tie-break, member symbols); each merge deepens its members.
    heap = [(int(freqs[s]), i, [s]) for i, s in enumerate(order)]
    heapq.heapify(heap)
    depth = {s: 0 for s in order}
    tie = len(order)
    while len(heap) > 1:
        fa, _, a = heapq.heappop(heap)
        fb, _, b = heapq.heappop(heap)
        for s in a + b:
            depth[s] += 1
        heapq.heappush(heap, (fa + fb, tie, a + b))
        tie += 1
    return depth


def canonical_codes(lengths):
    """{symbol: length} -> {symbol: (length, value)} in canonical order
    (shorter codes first, then real symbols by value, EOF last)."""
    order = sorted(lengths, key=lambda s: (lengths[s], isinstance(s, _EndOfFile),
                                           s if isinstance(s, int) else 0))
    table = {}
    code, prev = 0, None
    for s in order:
        n = lengths[s]
        if prev is not None:
            code = (code + 1) << (n - prev)
        table[s] = (n, code)
        prev = n
    return table


def huffman_code_table(frequencies):
    lengths = huffman_code_lengths(frequencies)
    if max(lengths.values()) > MAX_CODE_BITS:
        raise ValueError("code longer than 16 bits")
    return canonical_codes(lengths)


# ---------------------------------------------------------------------------
# utils.py counterparts
# ---------------------------------------------------------------------------

def flatten_block_of_weights(layers, dtype=torch.float8_e4m3fn):
    """Concatenates the weights of `layers` ({name: module}, in the order given)
    into one flat tensor; also returns the split positions (cumulative sizes
    without the last).  dfloat/utils.py:188-204."""
    sizes = [m.weight.numel() for m in layers.values()]
    flat = torch.empty(sum(sizes), dtype=dtype)
    off = 0
    for m, n in zip(layers.values(), sizes):
        flat[off:off + n] = m.weight.data.detach().reshape(-1)
        off += n
    split_positions = torch.cumsum(torch.tensor(sizes, dtype=torch.int64), 0)[:-1]
    return flat, split_positions


def repo_id_to_model_id(repo_id):
    """'org/name' -> 'models--org--name' (dfloat/utils.py:70-72)."""
    return "models--" + "--".join(repo_id.split("/"))


def locate_block_by_regex(model, pattern):
    """{full name: module} of every module whose name fully matches `pattern`
    (dfloat/utils.py:75-80)."""
    return {n: m for n, m in model.named_modules() if re.fullmatch(pattern, n)}


def _child_name(name, child):
    return f"{name}.{child}" if name else child


def find_layers_by_selection(module, select, name=""):
    """{full name: module} of the sub-modules at the dotted paths in `select`,
    looked up from `module` and from every module below it, sorted by name
    (dfloat/utils.py:83-117)."""
    res = {}
    for path in select:
        target = module
        try:
            for part in path.split("."):
                target = getattr(target, part)
        except AttributeError:
            continue
        res[_child_name(name, path)] = target
    for child_name, child in module.named_children():
        res.update(find_layers_by_selection(child, select, _child_name(name, child_name)))
    return dict(sorted(res.items()))


def find_layers_by_layer_type(module, layers=(torch.nn.Linear,), name=""):
    """The outermost modules whose exact type is in `layers`
    (dfloat/utils.py:120-132)."""
    if type(module) in tuple(layers):
        return {name: module}
    res = {}
    for child_name, child in module.named_children():
        res.update(find_layers_by_layer_type(child, layers, _child_name(name, child_name)))
    return dict(sorted(res.items()))


def _weight_dtype(module):
    w = getattr(module, "weight", None)
    return getattr(w, "dtype", None)


def find_layers_by_data_type(module, target_dtype=torch.bfloat16, name=""):
    """The outermost modules whose `weight` has `target_dtype`
    (dfloat/utils.py:135-155)."""
    if _weight_dtype(module) == target_dtype:
        return {name: module}
    res = {}
    for child_name, child in module.named_children():
        res.update(find_layers_by_data_type(child, target_dtype, _child_name(name, child_name)))
    return dict(sorted(res.items()))


def find_layers_by_data_type_and_layer_type(module, target_dtype=torch.bfloat16,
                                            layers=(torch.nn.Linear, torch.nn.Embedding), name=""):
    """The outermost modules of a type in `layers` whose `weight` has
    `target_dtype` (dfloat/utils.py:158-185)."""
    if type(module) in tuple(layers) and _weight_dtype(module) == target_dtype:
        return {name: module}
    res = {}
    for child_name, child in module.named_children():
        res.update(find_layers_by_data_type_and_layer_type(child, target_dtype, layers,
                                                           _child_name(name, child_name)))
    return dict(sorted(res.items()))


def get_exponents_and_other_4bits_fp8_e4m3(data):
    """e4m3 bytes `s eeee mmm` -> (exponents e, packed nibbles (s<<3|m) two per
    byte, even element in the high nibble).  dfloat/utils.py:207-227."""
    assert data.ndim == 1 and data.dtype == torch.float8_e4m3fn
    w = data.view(torch.uint8)
    exps = (w >> 3) & 0xF
    other = ((w >> 4) & 0x8) | (w & 0x7)
    pairs = other.view(-1, 2)
    return exps, (pairs[:, 0] << 4) | pairs[:, 1]


def compute_shannon_entropy(data):
    _, freqs = torch.unique(data, return_counts=True)
    p = freqs.double() / freqs.sum()
    return float(-(p * torch.log2(p)).sum())


def get_nbit_codec(counter, max_n_bits=MAX_CODE_BITS):
    """{symbol: count} -> (codec, counter, table), as dfloat/utils.py:239-267.
    With at most 16 symbols plus EOF every Huffman code fits in 16 bits."""
    if max_n_bits < MAX_CODE_BITS:
        raise ValueError("ECF8 streams allow codes of up to 16 bits")
    code = HuffmanCode.from_frequencies(counter)
    return code, counter, code.get_code_table()


def _fill_row(row, keys):
    """Byte-indexed row: each entry holds the value of the closest key at or
    below it, 0 before the first key (utils.py:352-357)."""
    cur = 0
    for b in range(256):
        cur = keys.get(b, cur)
        row[b] = cur


def _put(keys, key, val):
    if keys.get(key, val) != val:
        raise ValueError(f"LUT key {key} maps to both {keys[key]} and {val}")
    keys[key] = val


def get_luts_from_huffman_table(table):
    """Two-level byte LUTs of a code table (dfloat/utils.py:270-370 layout).

    Row 0 is indexed by the next stream byte.  Each code of up to 8 bits
    owns the key of its left-aligned bits; a longer code owns the key of its
    leading byte, whose value 256 - r points at row r.  Rows 1.. are those
    leading bytes in first-seen table order, indexed by the following byte.
    The last row maps a symbol to its code length.  The EOF symbol is left
    out.  Returns a uint8 tensor of shape (rows, 256).
    """
    codes = [(s, n, v) for s, (n, v) in table.items() if isinstance(s, (int, np.integer))
             and not isinstance(s, bool)]
    if any(n > MAX_CODE_BITS or n < 1 for _, n, _ in codes):
        raise ValueError("code lengths must be 1..16 bits")
    lead = []
    for _, n, v in codes:
        if n > 8 and (v >> (n - 8)) not in lead:
            lead.append(v >> (n - 8))
    luts = np.zeros((len(lead) + 2, 256), dtype=np.uint8)
    row0 = {}
    for s, n, v in codes:
        if n <= 8:
            _put(row0, v << (8 - n), int(s))
        else:
            _put(row0, v >> (n - 8), 256 - (1 + lead.index(v >> (n - 8))))
    _fill_row(luts[0], row0)
    for r, b in enumerate(lead, start=1):
        keys = {}
        for s, n, v in codes:
            if n > 8 and (v >> (n - 8)) == b:
                _put(keys, (v & ((1 << (n - 8)) - 1)) << (16 - n), int(s))
        _fill_row(luts[r], keys)
    for s, n, _ in codes:
        luts[-1, int(s)] = n
    return torch.from_numpy(luts)


def _code_arrays(codec):
    table = codec.get_code_table()
    eof = codec._eof
    bits = np.zeros(16, np.uint8)
    vals = np.zeros(16, np.uint32)
    for s, (n, v) in table.items():
        if s == eof or not isinstance(s, (int, np.integer)):
            continue
        if not 0 <= int(s) < 16:
            raise ValueError("ECF8 exponent symbols are 0..15")
        bits[int(s)] = n
        vals[int(s)] = v
    eb, ev = table[eof]
    return bits, vals, int(eb), int(ev)


def encode_exponents_for_cuda(exponents_4bits, codec, bytes_per_thread=8, threads_per_block=512):
    """Packs 4-bit exponents into (encoded u8, gaps u8, output_positions u64)
    exactly as dfloat/utils.py:502-530 does, on the GPU.  Tensors come back on
    the input's device (CPU input is packed on the current CUDA device)."""
    if bytes_per_thread != _lib.BYTES_PER_THREAD or threads_per_block != _lib.THREADS_PER_BLOCK:
        raise ValueError("only bytes_per_thread=8, threads_per_block=512 streams are supported")
    if not torch.cuda.is_available():
        raise RuntimeError("the ECF8 packer runs on a CUDA device")
    L = _lib.lib()
    home = exponents_4bits.device
    dev = home if home.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    ex = exponents_4bits.reshape(-1).to(device=dev, dtype=torch.uint8).contiguous()
    n = ex.numel()
    bits, vals, eof_bits, eof_val = _code_arrays(codec)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        ws = torch.empty(L.ecf8_encode_workspace_bytes(n), dtype=torch.uint8, device=dev)
        _lib.check(L.ecf8_encode_plan(ex.data_ptr(), n, bits.tobytes(), eof_bits, ws.data_ptr(), stream),
                   "ecf8_encode_plan")
        invalid, total_bits, n_bytes, n_op = (int(x) for x in ws[-32:].view(torch.int64).cpu().tolist())
        if invalid:
            raise ValueError(f"{invalid} exponents are above 15 or have no code")
        group = bytes_per_thread * threads_per_block
        grid = -(-n_bytes // group)
        cap = (n_bytes + 15) & ~15
        encoded = torch.empty(max(cap, 16), dtype=torch.uint8, device=dev)
        gaps = torch.empty(max(grid * threads_per_block // 2, 4), dtype=torch.uint8, device=dev)
        op = torch.empty(n_op, dtype=torch.int64, device=dev)
        cvals = (ctypes.c_uint32 * 16)(*[int(x) for x in vals])
        _lib.check(L.ecf8_encode_emit(ex.data_ptr(), n, bits.tobytes(), cvals, eof_bits, eof_val,
                                      ws.data_ptr(), encoded.data_ptr(), n_bytes, encoded.numel(),
                                      gaps.data_ptr(), grid * threads_per_block // 2, op.data_ptr(),
                                      n_op, stream), "ecf8_encode_emit")
        encoded = encoded[:n_bytes].clone()
        gaps = gaps[:grid * threads_per_block // 2].clone()
        op = op.view(torch.uint64)
    del total_bits
    if home.type != "cuda":
        encoded, gaps, op = encoded.cpu(), gaps.cpu(), op.cpu()
    return encoded, gaps, op


def compress_fp8(flat, device=None):
    """Compresses one flat e4m3 tensor into the five ECF8 stream buffers
    (luts, encoded, packed_other_4bits, output_positions, gaps), the same set
    the reference compressor stores per block (scripts/compress.py:239-247).
    Runs on `device` (default: the tensor's device, or the current GPU)."""
    if device is None:
        device = flat.device if flat.device.type == "cuda" else torch.device("cuda")
    flat = flat.reshape(-1).to(device)
    exps, packed = get_exponents_and_other_4bits_fp8_e4m3(flat)
    counts = torch.bincount(exps.long(), minlength=16).cpu().tolist()
    counter = {s: c for s, c in enumerate(counts) if c > 0}
    codec, _, table = get_nbit_codec(counter)
    luts = get_luts_from_huffman_table(table).to(device)
    encoded, gaps, op = encode_exponents_for_cuda(exps, codec)
    entropy = -sum((c / flat.numel()) * math.log2(c / flat.numel()) for c in counter.values())
    return {
        "luts": luts,
        "encoded": encoded,
        "packed_other_4bits": packed.contiguous(),
        "output_positions": op,
        "gaps": gaps,
        "entropy": entropy,
        "table": table,
    }
