"""Generates the golden ECF8 streams under tests/golden/ from the REFERENCE codec.

Run where a reference checkout exists, named by ECF8_REFERENCE_DIR:

    ECF8_REFERENCE_DIR=/path/to/ecf8 python tests/golden/make_fixtures.py

It imports the reference's own ``dfloat/utils.py`` (with the test-only
``oracle/dahuffman.py`` stand-in for the missing third-party ``dahuffman``)
and records, per case, the original e4m3 bytes plus everything the reference
compressor stores for a block (scripts/compress.py:239-247): the LUTs
(utils.py:270-370), the exponent bitstream, packed gaps and output positions
(utils.py:373-499) and the packed sign+mantissa nibbles (utils.py:207-227),
together with the code table the LUTs were built from.  Decoding those
buffers must give back the original bytes.

Config 1 of the benchmark spec (a 4096x4096 N(0, 0.02) tensor, seed 0,
per-tensor absmax->448) is too large to commit, so only SHA-256 digests of
its reference-encoded buffers are stored (config1_digests.json); tests
regenerate the tensor with the same seeded torch generator and compare.
Nothing at test time reads the reference checkout.
"""

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("ECF8_REFERENCE_DIR")
if not REF or not os.path.isfile(os.path.join(REF, "dfloat", "utils.py")):
    sys.exit("make_fixtures.py: set ECF8_REFERENCE_DIR to a zeyuyang8/ecf8 checkout")
sys.path.insert(0, os.path.join(REPO, "oracle"))  # dahuffman stand-in
sys.path.insert(0, REF)

from dahuffman import HuffmanCodec  # noqa: E402  (oracle/dahuffman.py)
from dfloat import utils as U  # noqa: E402  (the reference codec)

TPB, BPT = 512, 8


def fp8_bytes_from_fields(exps, rng):
    """e4m3 bytes with the given exponents and random sign/mantissa bits."""
    n = exps.size
    sign = rng.integers(0, 2, n, dtype=np.uint8)
    mant = rng.integers(0, 8, n, dtype=np.uint8)
    return ((sign << 7) | (exps.astype(np.uint8) << 3) | mant).astype(np.uint8)


def table_arrays(table, eof):
    """The code table in its dict order: (symbols, bits, values, eof_bits, eof_val)."""
    syms, bits, vals = [], [], []
    for s, (b, v) in table.items():
        if s == eof or not isinstance(s, int):
            continue
        syms.append(s)
        bits.append(b)
        vals.append(v)
    eb, ev = table[eof]
    return (np.array(syms, np.int32), np.array(bits, np.int32),
            np.array(vals, np.int64), np.int32(eb), np.int64(ev))


def encode_reference(fp8_u8, codec=None):
    """Runs the reference codec on e4m3 bytes; returns a dict of arrays."""
    flat = torch.from_numpy(fp8_u8.copy()).view(torch.float8_e4m3fn)
    exps, packed = U.get_exponents_and_other_4bits_fp8_e4m3(flat)
    if codec is None:
        vals, freqs = torch.unique(exps, return_counts=True)
        counter = {v: f for v, f in zip(vals.tolist(), freqs.tolist())}
        codec, _, table = U.get_nbit_codec(counter, max_n_bits=16)
    table = codec.get_code_table()
    luts = U.get_luts_from_huffman_table(table)
    encoded, gaps, op = U.encode_exponents_for_cuda(exps, codec, BPT, TPB)
    syms, bits, vals, eb, ev = table_arrays(table, codec._eof)
    return {
        "fp8": fp8_u8.astype(np.uint8),
        "luts": luts.numpy().astype(np.uint8),
        "encoded": encoded.numpy().astype(np.uint8),
        "packed": packed.numpy().astype(np.uint8),
        "gaps": gaps.numpy().astype(np.uint8),
        "output_positions": op.numpy().astype(np.uint64),
        "table_symbols": syms,
        "table_bits": bits,
        "table_values": vals,
        "eof_bits": eb,
        "eof_value": ev,
        "threads_per_block": np.int32(TPB),
        "bytes_per_thread": np.int32(BPT),
    }


def quantize_per_tensor(w):
    scale = 448.0 / w.abs().max()
    return (w * scale).to(torch.float8_e4m3fn).view(torch.uint8).flatten().numpy()


def quantize_block_128(w):
    out, inn = w.shape
    t = w.reshape(out // 128, 128, inn // 128, 128)
    amax = t.abs().amax(dim=(1, 3), keepdim=True).clamp(min=1e-12)
    q = (t * (448.0 / amax)).to(torch.float8_e4m3fn)
    return q.reshape(out, inn).view(torch.uint8).flatten().numpy()


def custom_codec(codes, eof_code):
    """A HuffmanCodec-shaped object for an explicit prefix code {sym: bitstring}."""
    table = {s: (len(c), int(c, 2)) for s, c in codes.items()}
    eof = HuffmanCodec.from_frequencies({0: 1})._eof
    table[eof] = (len(eof_code), int(eof_code, 2))
    return HuffmanCodec(table, eof=eof)


def long_code_codec():
    """Symbol 0 gets the 1-bit code '0'; symbols 1..15 get 16-bit codes under
    fifteen distinct 8-bit prefixes (a 17-row LUT).  Mixing the two puts
    16-bit codes at every bit offset, so gaps reach 15."""
    codes = {0: "0"}
    for s in range(1, 16):
        prefix = format(0x80 | (s * 7 % 128), "08b")
        codes[s] = prefix + format((s * 37) % 256, "08b")
    eof = format(0x80 | 127, "08b") + "11111111"
    return custom_codec(codes, eof)


def max_lut_codec():
    """All sixteen symbols get 16-bit codes under sixteen distinct first
    bytes: the LUT reaches its maximum of 18 rows (row 0, sixteen prefix
    rows, the length row)."""
    codes = {s: format(s * 16, "08b") + format((s * 91) % 256, "08b")
             for s in range(16)}
    return custom_codec(codes, format(0x0F, "08b") + "11111111")


def cases():
    rng = np.random.default_rng(2024)
    g = torch.Generator().manual_seed(1)
    out = {}
    # Trained-weight-like exponent statistics, per-tensor scale.
    out["gauss_per_tensor"] = encode_reference(
        quantize_per_tensor(torch.randn(1024, 192, generator=g) * 0.02))
    # 128x128 block scales, as in the Qwen3-shaped configs.
    out["gauss_block128"] = encode_reference(
        quantize_block_128(torch.randn(256, 512, generator=g) * 0.02))
    # A symbol with more than half the mass gets a 1-bit code.
    e = rng.choice(16, size=120_000, p=np.r_[[0.7], np.full(15, 0.3 / 15)])
    out["one_bit_code"] = encode_reference(fp8_bytes_from_fields(e, rng))
    # Fibonacci frequencies: the Huffman tree reaches depth 16.
    fib = [1, 1]
    while len(fib) < 16:
        fib.append(fib[-1] + fib[-2])
    p = np.array(fib[::-1], np.float64)
    e = rng.choice(16, size=150_000, p=p / p.sum())
    out["fibonacci_depth16"] = encode_reference(fp8_bytes_from_fields(e, rng))
    # Explicit code: 16-bit codes everywhere (gaps up to 15), n_luts = 18.
    e = rng.choice(16, size=40_000, p=np.r_[[0.25], np.full(15, 0.75 / 15)])
    out["sixteen_bit_codes"] = encode_reference(
        fp8_bytes_from_fields(e, rng), codec=long_code_codec())
    e = rng.choice(16, size=20_000)
    out["max_luts_18"] = encode_reference(
        fp8_bytes_from_fields(e, rng), codec=max_lut_codec())
    # Only exponent 0: 1-bit codes, 32768 elements per group.
    e = np.zeros(70_000, np.int64)
    out["single_symbol_zero"] = encode_reference(fp8_bytes_from_fields(e, rng))
    # Only exponent 7: the reference kernel would spin on the EOF bits
    # (length-0 code); oracle and product must still decode it.
    e = np.full(5_000, 7, np.int64)
    out["single_symbol_seven"] = encode_reference(fp8_bytes_from_fields(e, rng))
    # Tiny streams: one partial window / group.
    for n in (2, 6, 16, 30, 130):
        e = rng.choice(16, size=n)
        out[f"tiny_{n}"] = encode_reference(fp8_bytes_from_fields(e, rng))
    # A stream whose bit length is a multiple of 8 (no EOF byte appended).
    base = rng.choice(16, size=5_000, p=np.r_[[0.5], np.full(15, 0.5 / 15)])
    for n in range(4_000, 5_000, 2):
        r = encode_reference(fp8_bytes_from_fields(base[:n], rng))
        bits = dict(zip(r["table_symbols"].tolist(), r["table_bits"].tolist()))
        total = sum(bits[int(x)] for x in base[:n])
        if total % 8 == 0:
            out["byte_aligned_end"] = r
            break
    # The last code straddles a group boundary and the stream ends on a byte
    # boundary one byte into the new group: output_positions then has one
    # entry fewer than the decode grid + 1.
    out["op_short_by_one"] = encode_reference(*group_spill_case(rng))
    return out


def group_spill_case(rng):
    """2047 16-bit codes and 8 one-bit codes in random order, then a final
    16-bit code starting at bit 32760: 32776 bits in all, so the stream is
    4097 bytes (two decode groups) and no code starts in the second group."""
    codec = long_code_codec()
    head = np.r_[rng.integers(1, 16, 2047), np.zeros(8, np.int64)]
    rng.shuffle(head)
    e = np.r_[head, [int(rng.integers(1, 16))]].astype(np.int64)
    table = codec.get_code_table()
    assert sum(table[int(s)][0] for s in e) == 32768 + 8 and e.size % 2 == 0
    return fp8_bytes_from_fields(e, rng), codec


def config1():
    w = torch.randn(4096, 4096, generator=torch.Generator().manual_seed(0)) * 0.02
    r = encode_reference(quantize_per_tensor(w))
    dig = {k: hashlib.sha256(np.ascontiguousarray(r[k]).tobytes()).hexdigest()
           for k in ("fp8", "luts", "encoded", "packed", "gaps", "output_positions")}
    sizes = {k: int(r[k].size) for k in ("encoded", "gaps", "output_positions")}
    meta = {
        "config": "4096x4096 N(0,0.02) fp32, torch.Generator().manual_seed(0), "
                  "per-tensor scale 448/absmax, cast to float8_e4m3fn",
        "sha256": dig,
        "sizes": sizes,
        "table_symbols": r["table_symbols"].tolist(),
        "table_bits": r["table_bits"].tolist(),
        "table_values": r["table_values"].tolist(),
        "eof_bits": int(r["eof_bits"]),
        "eof_value": int(r["eof_value"]),
        "exponent_counts": np.bincount((r["fp8"] >> 3) & 0xF, minlength=16).tolist(),
    }
    return meta


def main():
    for name, arrs in cases().items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)
        print(name, {k: v.shape for k, v in arrs.items() if hasattr(v, "shape") and v.ndim})
    meta = config1()
    with open(os.path.join(HERE, "config1_digests.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("config1", meta["sizes"])


if __name__ == "__main__":
    main()
