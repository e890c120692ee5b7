"""Product codec (code tables, LUT builder) against the reference format."""
import numpy as np
import pytest

from conftest import golden_names, load_golden
from helpers import random_stream


def table_from_golden(s):
    from ecf8_b200.codec import EOF
    t = {int(a): (int(b), int(c)) for a, b, c in zip(s["table_symbols"], s["table_bits"], s["table_values"])}
    t[EOF] = (int(s["eof_bits"]), int(s["eof_value"]))
    return t


@pytest.mark.parametrize("name", golden_names())
def test_lut_builder_matches_reference(name):
    from ecf8_b200.codec import get_luts_from_huffman_table
    s = load_golden(name)
    luts = get_luts_from_huffman_table(table_from_golden(s)).numpy()
    assert luts.dtype == np.uint8
    assert np.array_equal(luts, s["luts"])


def test_lut_builder_rejects_conflicting_codes():
    from ecf8_b200.codec import EOF, get_luts_from_huffman_table
    with pytest.raises(ValueError):
        get_luts_from_huffman_table({1: (2, 1), 2: (2, 1), EOF: (2, 3)})


@pytest.mark.parametrize("seed", range(20))
def test_product_code_tables_are_valid_and_safe(oracle_mod, seed):
    from ecf8_b200 import codec
    rng = np.random.default_rng(seed)
    k = int(rng.integers(1, 17))
    cnt = {int(s): int(c) for s, c in zip(rng.choice(16, k, replace=False),
                                          rng.integers(1, 10 ** 6, k))}
    table = codec.huffman_code_table(cnt)
    assert set(table) == set(cnt) | {codec.EOF}
    lens = [b for b, _ in table.values()]
    assert max(lens) <= 16
    assert abs(sum(2.0 ** -b for b in lens) - 1.0) < 1e-12  # complete prefix code
    codes = [format(v, f"0{b}b") for b, v in table.values()]
    for a in codes:
        for b in codes:
            assert a == b or not b.startswith(a)
    luts = codec.get_luts_from_huffman_table(table).numpy()
    # canonical codes leave no LUT path that yields a length-0 code
    assert oracle_mod.reference_kernel_terminates(luts)


def test_huffman_is_optimal_on_config1_counts():
    import json, os
    from conftest import GOLDEN
    from ecf8_b200 import codec
    meta = json.load(open(os.path.join(GOLDEN, "config1_digests.json")))
    cnt = {s: c for s, c in enumerate(meta["exponent_counts"]) if c}
    mine = codec.huffman_code_table(cnt)
    ref_bits = dict(zip(meta["table_symbols"], meta["table_bits"]))
    cost = lambda bits: sum(cnt[s] * bits[s] for s in cnt)
    # both are Huffman codes: same total length (ties may assign lengths differently)
    assert cost({s: mine[s][0] for s in cnt}) == cost(ref_bits)


@pytest.mark.parametrize("seed", range(8))
def test_random_streams_round_trip_through_oracle(oracle_mod, seed):
    rng = np.random.default_rng(100 + seed)
    s = random_stream(oracle_mod, rng)
    out, zl = oracle_mod.decode(s)
    assert zl == 0
    assert np.array_equal(out, s["fp8"])


def test_exponent_split_matches_reference_layout(oracle_mod):
    import torch
    from ecf8_b200.codec import get_exponents_and_other_4bits_fp8_e4m3
    s = load_golden("gauss_block128")
    t = torch.from_numpy(s["fp8"].copy()).view(torch.float8_e4m3fn)
    e, p = get_exponents_and_other_4bits_fp8_e4m3(t)
    oe, op_ = oracle_mod.split(s["fp8"])
    assert np.array_equal(e.numpy(), oe) and np.array_equal(p.numpy(), s["packed"])


def test_flatten_block_of_weights_order_and_splits():
    import torch
    from ecf8_b200.codec import flatten_block_of_weights
    a = torch.nn.Linear(4, 3, bias=False)
    b = torch.nn.Linear(2, 5, bias=False)
    for m in (a, b):
        m.weight.data = m.weight.data.to(torch.float8_e4m3fn)
    flat, split = flatten_block_of_weights({"a": a, "b": b})
    assert flat.numel() == 22 and split.tolist() == [12]
    assert torch.equal(flat[:12].view(torch.uint8), a.weight.data.reshape(-1).view(torch.uint8))
