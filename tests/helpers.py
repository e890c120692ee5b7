"""Shared test helpers: synthetic streams built with the product code tables
and the oracle packer (a restatement of the reference packer)."""
import numpy as np
import torch


def fp8_from_exponents(e, rng):
    n = e.size
    return ((rng.integers(0, 2, n).astype(np.uint8) << 7) | (e.astype(np.uint8) << 3)
            | rng.integers(0, 8, n).astype(np.uint8)).astype(np.uint8)


def table_to_arrays(table):
    from ecf8_b200.codec import EOF
    bits = np.zeros(16, np.uint8)
    vals = np.zeros(16, np.uint32)
    for s, (b, v) in table.items():
        if isinstance(s, int):
            bits[s] = b
            vals[s] = v
    eb, ev = table[EOF]
    return bits, vals, int(eb), int(ev)


def random_stream(oracle, rng, n=None, k=None, alpha=None):
    """A random stream (dict of numpy arrays + original bytes) whose code
    table comes from the product Huffman builder and whose bitstream comes
    from the oracle packer."""
    from ecf8_b200 import codec
    k = int(rng.integers(1, 17)) if k is None else k
    syms = rng.choice(16, size=k, replace=False)
    alpha = float(rng.choice([0.05, 0.3, 1.0, 5.0])) if alpha is None else alpha
    p = rng.dirichlet(np.full(k, alpha))
    n = int(rng.integers(1, 60000)) * 2 if n is None else n
    e = rng.choice(syms, size=n, p=p).astype(np.uint8)
    cnt = {int(s): int(c) for s, c in zip(*np.unique(e, return_counts=True))}
    table = codec.huffman_code_table(cnt)
    luts = codec.get_luts_from_huffman_table(table).numpy()
    bits, vals, eb, ev = table_to_arrays(table)
    enc, gaps, op = oracle.encode(e, bits, vals, eb, ev)
    fp8 = fp8_from_exponents(e, rng)
    _, packed = oracle.split(fp8)
    return {"fp8": fp8, "luts": luts, "encoded": enc, "packed": packed, "gaps": gaps,
            "output_positions": op, "table": table}


def to_device(s, device):
    return {
        "luts": torch.from_numpy(np.ascontiguousarray(s["luts"])).to(device),
        "encoded": torch.from_numpy(np.ascontiguousarray(s["encoded"])).to(device),
        "packed_other_4bits": torch.from_numpy(np.ascontiguousarray(s["packed"])).to(device),
        "output_positions": torch.from_numpy(np.ascontiguousarray(s["output_positions"]).view(np.int64)).to(device),
        "gaps": torch.from_numpy(np.ascontiguousarray(s["gaps"])).to(device),
    }
