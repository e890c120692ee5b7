"""The oracle (C restatement of the reference decode kernel and packer) is
pinned against golden vectors produced by the reference codec itself."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_names, load_golden


@pytest.mark.parametrize("name", golden_names())
def test_oracle_decode_matches_original(oracle_mod, name):
    s = load_golden(name)
    out, zero_len = oracle_mod.decode(s)
    assert np.array_equal(out, s["fp8"])
    # the reference kernel terminates exactly when no zero-length code is met
    if oracle_mod.reference_kernel_terminates(s["luts"]):
        assert zero_len == 0


@pytest.mark.parametrize("name", golden_names())
def test_oracle_packer_matches_reference_packer(oracle_mod, name):
    s = load_golden(name)
    bits, vals = oracle_mod.table_arrays(s["table_symbols"], s["table_bits"], s["table_values"])
    e, p = oracle_mod.split(s["fp8"])
    enc, gaps, op = oracle_mod.encode(e, bits, vals, int(s["eof_bits"]), int(s["eof_value"]))
    assert np.array_equal(p, s["packed"])
    assert np.array_equal(enc, s["encoded"])
    assert np.array_equal(gaps, s["gaps"])
    assert np.array_equal(op, s["output_positions"])


def test_single_symbol_seven_would_spin_the_reference(oracle_mod):
    s = load_golden("single_symbol_seven")
    assert not oracle_mod.reference_kernel_terminates(s["luts"])
    out, zero_len = oracle_mod.decode(s)
    assert zero_len > 0 and np.array_equal(out, s["fp8"])


def test_short_output_positions_case(oracle_mod):
    s = load_golden("op_short_by_one")
    grid = -(-s["encoded"].size // 4096)
    assert s["output_positions"].size == grid  # one fewer than the reference kernel reads


def config1_fp8():
    w = torch.randn(4096, 4096, generator=torch.Generator().manual_seed(0)) * 0.02
    scale = 448.0 / w.abs().max()
    return (w * scale).to(torch.float8_e4m3fn).view(torch.uint8).flatten().numpy()


def test_config1_cpu_round_trip(oracle_mod):
    """Config 1: 4096x4096 N(0,0.02), per-tensor scale, encoded with the
    reference's code table; buffers must hash like the reference packer's and
    decode back bit-exactly on the CPU."""
    meta = json.load(open(os.path.join(GOLDEN, "config1_digests.json")))
    fp8 = config1_fp8()
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    assert sha(fp8) == meta["sha256"]["fp8"]
    bits, vals = oracle_mod.table_arrays(meta["table_symbols"], meta["table_bits"], meta["table_values"])
    e, packed = oracle_mod.split(fp8)
    enc, gaps, op = oracle_mod.encode(e, bits, vals, meta["eof_bits"], meta["eof_value"])
    assert sha(packed) == meta["sha256"]["packed"]
    assert sha(enc) == meta["sha256"]["encoded"]
    assert sha(gaps) == meta["sha256"]["gaps"]
    assert sha(op) == meta["sha256"]["output_positions"]
    counts = np.bincount(e, minlength=16)
    assert counts.tolist() == meta["exponent_counts"]
    p = counts[counts > 0] / counts.sum()
    assert abs(-(p * np.log2(p)).sum() - 2.544) < 0.001
    from ecf8_b200.codec import EOF, get_luts_from_huffman_table
    table = {int(s): (int(b), int(v)) for s, b, v in
             zip(meta["table_symbols"], meta["table_bits"], meta["table_values"])}
    table[EOF] = (meta["eof_bits"], meta["eof_value"])
    luts = get_luts_from_huffman_table(table).numpy()
    assert sha(luts) == meta["sha256"]["luts"]
    out, zl = oracle_mod.decode({"luts": luts, "encoded": enc, "packed": packed, "gaps": gaps,
                                 "output_positions": op})
    assert np.array_equal(out, fp8)


@pytest.mark.parametrize("name", golden_names())
def test_oracle_lut_restatement_matches_reference(oracle_mod, name):
    s = load_golden(name)
    table = {int(a): (int(b), int(c)) for a, b, c in zip(s["table_symbols"], s["table_bits"], s["table_values"])}
    assert np.array_equal(oracle_mod.luts_from_table(table), s["luts"])


def test_dahuffman_standin_gives_complete_prefix_codes():
    from dahuffman import HuffmanCodec
    rng = np.random.default_rng(5)
    for _ in range(20):
        k = int(rng.integers(1, 17))
        freqs = {int(s): int(f) for s, f in zip(rng.choice(16, k, replace=False), rng.integers(1, 10 ** 6, k))}
        t = HuffmanCodec.from_frequencies(freqs).get_code_table()
        assert len(t) == k + 1
        assert abs(sum(2.0 ** -b for b, _ in t.values()) - 1.0) < 1e-12
        assert max(b for b, _ in t.values()) <= 16


def test_oracle_decodes_codes_up_to_16_bits(oracle_mod):
    """Power-of-two counts give codes of 1 to 16 bits (the longest take both
    LUT levels); with the data drawn uniformly the oracle still restores the
    original bytes."""
    from ecf8_b200 import codec
    from helpers import fp8_from_exponents, table_to_arrays
    rng = np.random.default_rng(11)
    table = codec.huffman_code_table({int(s): 1 << i for i, s in enumerate(rng.permutation(16))})
    bits, vals, eb, ev = table_to_arrays(table)
    assert bits.max() == 16
    e = rng.integers(0, 16, 100000).astype(np.uint8)
    enc, gaps, op = oracle_mod.encode(e, bits, vals, eb, ev)
    fp8 = fp8_from_exponents(e, rng)
    _, packed = oracle_mod.split(fp8)
    s = {"luts": codec.get_luts_from_huffman_table(table).numpy(), "encoded": enc, "packed": packed,
         "gaps": gaps, "output_positions": op}
    out, _ = oracle_mod.decode(s)
    assert np.array_equal(out, fp8)
