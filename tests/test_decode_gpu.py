"""GPU parity: the sm_100a decode kernel (through the C ABI) against the
original bytes, the CPU oracle and the reference kernel decode.cu compiled
unmodified for sm_100a, on the reference's own golden streams, adversarial
streams and random streams."""
import hashlib
import json
import math
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_names, load_golden
from helpers import random_stream, to_device

pytestmark = pytest.mark.gpu
GUARD = 0xA5


def decode_guarded(d, n, dev, offset=0, misalign=False):
    """Decodes into the middle of a guard-filled buffer; returns (decoded,
    guard bytes).  misalign=True shifts every input and the output by one byte
    so the kernel's unaligned path runs."""
    from ecf8_b200.run import decode_stream
    if misalign:  # output_positions must stay 8-byte aligned (the ABI rejects it otherwise)
        d = {k: (_shift(v) if k in ("encoded", "packed_other_4bits", "gaps") else v) for k, v in d.items()}
    off = 33 if misalign else 32
    buf = torch.full((n + 64,), GUARD, dtype=torch.uint8, device=dev)
    out = buf[off:off + n]
    decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"], out)
    torch.cuda.synchronize()
    b = buf.cpu().numpy()
    return b[off:off + n], np.concatenate([b[:off], b[off + n:]])


def _shift(t):
    big = torch.empty(t.numel() + 1, dtype=torch.uint8, device=t.device)
    big[1:] = t
    return big[1:]


def run_reference_kernel(s, dev):
    """The reference kernel on the same stream (dfloat/run/run.py:97-119
    geometry).  The LUT buffer is padded to 18 rows and output_positions by
    one trailing n_elements entry so its reads past the arrays stay inside."""
    import oracle
    L = oracle.ref_lib()
    n = s["packed"].size * 2
    luts = np.zeros((18, 256), np.uint8)
    luts[:s["luts"].shape[0]] = s["luts"]
    op = np.concatenate([s["output_positions"], np.array([n], np.uint64)])
    t = {"luts": torch.from_numpy(luts).to(dev), "enc": torch.from_numpy(s["encoded"].copy()).to(dev),
         "packed": torch.from_numpy(s["packed"].copy()).to(dev),
         "op": torch.from_numpy(op.view(np.int64).copy()).to(dev),
         "gaps": torch.from_numpy(s["gaps"].copy()).to(dev)}
    out = torch.zeros(n, dtype=torch.uint8, device=dev)
    grid = math.ceil(s["encoded"].size / 4096)
    per = np.diff(s["output_positions"].astype(np.int64))
    smem = 512 * 4 + 4 + int(per.max() if per.size else 0)
    st = L.ref_decode_launch(t["luts"].data_ptr(), t["enc"].data_ptr(), t["packed"].data_ptr(),
                             t["op"].data_ptr(), t["gaps"].data_ptr(), out.data_ptr(),
                             s["luts"].shape[0], s["encoded"].size, n, grid, 512, smem,
                             torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("name", golden_names())
@pytest.mark.parametrize("misalign", [False, True])
def test_golden_streams(cuda_device, oracle_mod, name, misalign):
    s = load_golden(name)
    dec, guard = decode_guarded(to_device(s, cuda_device), s["fp8"].size, cuda_device, misalign=misalign)
    assert np.all(guard == GUARD), "wrote outside outputs[0, n)"
    assert np.array_equal(dec, s["fp8"])
    ora, _ = oracle_mod.decode(s)
    assert np.array_equal(dec, ora)


@pytest.mark.parametrize("name", golden_names())
def test_golden_streams_match_reference_kernel(cuda_device, oracle_mod, name):
    s = load_golden(name)
    if not oracle_mod.reference_kernel_terminates(s["luts"]):
        pytest.skip("the reference kernel spins on this stream's EOF bits")
    ref = run_reference_kernel(s, cuda_device)
    dec, _ = decode_guarded(to_device(s, cuda_device), s["fp8"].size, cuda_device)
    assert np.array_equal(ref, s["fp8"])
    assert np.array_equal(dec, ref)


@pytest.mark.parametrize("seed", range(40))
def test_random_streams(cuda_device, oracle_mod, seed):
    rng = np.random.default_rng(1000 + seed)
    s = random_stream(oracle_mod, rng)
    dec, guard = decode_guarded(to_device(s, cuda_device), s["fp8"].size, cuda_device)
    assert np.all(guard == GUARD)
    assert np.array_equal(dec, s["fp8"])
    if seed % 4 == 0:
        assert np.array_equal(run_reference_kernel(s, cuda_device), dec)


@pytest.mark.parametrize("k,misalign", [(1, False), (2, False), (2, True), (3, False)])
def test_highly_compressible_groups(cuda_device, oracle_mod, k, misalign):
    """Streams of one to three symbols: codes of about one bit put up to
    32768 elements in a 4096-byte group, more than one pass of the kernel's
    16384-element output window."""
    rng = np.random.default_rng(50 + k)
    s = random_stream(oracle_mod, rng, n=300000, k=k, alpha=0.05)
    per = np.diff(np.append(s["output_positions"].astype(np.int64), s["fp8"].size))
    assert per.max() > 16384  # the multi-window path runs
    dec, guard = decode_guarded(to_device(s, cuda_device), s["fp8"].size, cuda_device, misalign=misalign)
    assert np.all(guard == GUARD)
    assert np.array_equal(dec, s["fp8"])


def test_highly_compressible_groups_with_prepared_table(cuda_device, oracle_mod):
    from ecf8_b200.run import build_decode_table, decode_stream
    rng = np.random.default_rng(61)
    s = random_stream(oracle_mod, rng, n=300000, k=2, alpha=0.05)
    d = to_device(s, cuda_device)
    out = torch.zeros(s["fp8"].size, dtype=torch.uint8, device=cuda_device)
    decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"], out,
                  table=build_decode_table(d["luts"]))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), s["fp8"])


def test_batch_of_all_golden_streams(cuda_device):
    from ecf8_b200.run import decode_streams
    names = golden_names()
    ss = [load_golden(n) for n in names]
    ds = [to_device(s, cuda_device) for s in ss]
    outs = [torch.zeros(s["fp8"].size, dtype=torch.uint8, device=cuda_device) for s in ss]
    decode_streams(ds, outs)
    torch.cuda.synchronize()
    for n, s, o in zip(names, ss, outs):
        assert np.array_equal(o.cpu().numpy(), s["fp8"]), n


@pytest.mark.parametrize("overlap", [False, True])
def test_batch_larger_than_one_launch(cuda_device, oracle_mod, overlap):
    """300 streams: two launches per call; with overlap the second may start while
    the one before it runs (their outputs are disjoint, their inputs were
    written before the call)."""
    from ecf8_b200.run import decode_streams
    rng = np.random.default_rng(7)
    ss = [random_stream(oracle_mod, rng, n=int(rng.integers(1, 3000)) * 2) for _ in range(300)]
    ds = [to_device(s, cuda_device) for s in ss]
    outs = [torch.zeros(s["fp8"].size, dtype=torch.uint8, device=cuda_device) for s in ss]
    torch.cuda.synchronize()
    decode_streams(ds, outs, overlap_previous=overlap)
    torch.cuda.synchronize()
    for s, o in zip(ss, outs):
        assert np.array_equal(o.cpu().numpy(), s["fp8"])


@pytest.mark.parametrize("ctas", [1, 3, 37])
def test_decode_with_fewer_ctas(cuda_device, oracle_mod, ctas):
    """ECF8_DECODE_CTAS(n): a launch of n CTAs (each covering more groups and
    more stream boundaries) gives the same bytes, with and without launch
    overlap, for a multi-stream batch and for a stream larger than the grid's
    share of work."""
    from ecf8_b200 import _lib
    from ecf8_b200.run import _stream_struct, build_decode_table, decode_stream
    rng = np.random.default_rng(ctas)
    ss = [random_stream(oracle_mod, rng, n=int(rng.integers(1, 4000)) * 2) for _ in range(9)]
    ss += [load_golden(n) for n in golden_names()[:4]]
    ds = [to_device(s, cuda_device) for s in ss]
    outs = [torch.full((s["fp8"].size,), GUARD, dtype=torch.uint8, device=cuda_device) for s in ss]
    for d in ds:
        d["decode_table"] = build_decode_table(d["luts"])
    arr = (_lib.Ecf8Stream * len(ds))(*[_stream_struct(d, o, d["decode_table"]) for d, o in zip(ds, outs)])
    L = _lib.lib()
    for flags in (_lib.decode_ctas(ctas), _lib.decode_ctas(ctas) | _lib.DECODE_OVERLAP_PREVIOUS):
        for o in outs:
            o.fill_(GUARD)
        st = L.ecf8_decode_batch_flags(arr, len(ds), 512, 8, flags, torch.cuda.current_stream().cuda_stream)
        assert st == _lib.OK
        torch.cuda.synchronize()
        for s, o in zip(ss, outs):
            assert np.array_equal(o.cpu().numpy(), s["fp8"])
    big = random_stream(oracle_mod, rng, n=400_000)
    d = to_device(big, cuda_device)
    out = decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"],
                        max_ctas=ctas)
    torch.cuda.synchronize()
    assert np.array_equal(out.view(torch.uint8).cpu().numpy(), big["fp8"])


def test_reference_call_convention(cuda_device):
    """`_decode(grid=, block=, shared_mem=, args=[...])` as compress.py:109-124 calls it."""
    from ecf8_b200 import _decode
    s = load_golden("gauss_per_tensor")
    d = to_device(s, cuda_device)
    n = s["fp8"].size
    out = torch.empty(n, dtype=torch.float8_e4m3fn, device=cuda_device)
    grid = (int(np.ceil(d["encoded"].numel() / (512 * 8))),)
    _decode(grid=grid, block=(512,), shared_mem=512 * 4 + 4 + 99999,
            args=[d["luts"].data_ptr(), d["encoded"].data_ptr(), d["packed_other_4bits"].data_ptr(),
                  d["output_positions"].data_ptr(), d["gaps"].data_ptr(), out.data_ptr(),
                  d["luts"].shape[0], d["encoded"].numel(), n])
    torch.cuda.synchronize()
    assert np.array_equal(out.view(torch.uint8).cpu().numpy(), s["fp8"])


def test_repeat_decode_is_idempotent(cuda_device):
    s = load_golden("fibonacci_depth16")
    d = to_device(s, cuda_device)
    a, _ = decode_guarded(d, s["fp8"].size, cuda_device)
    b, _ = decode_guarded(d, s["fp8"].size, cuda_device)
    assert np.array_equal(a, b)


def test_corrupt_streams_stay_in_bounds(cuda_device):
    """Garbage gaps / output positions / LUTs must not make the kernel touch
    memory outside the buffers it was given (unspecified bytes inside)."""
    rng = np.random.default_rng(3)
    s = load_golden("gauss_block128")
    n = s["fp8"].size
    for trial in range(6):
        c = {k: v.copy() for k, v in s.items()}
        if trial % 3 == 0:
            c["gaps"] = rng.integers(0, 256, c["gaps"].size).astype(np.uint8)
        elif trial % 3 == 1:
            c["output_positions"] = rng.integers(0, 2 * n, c["output_positions"].size).astype(np.uint64)
        else:
            c["luts"] = rng.integers(0, 256, c["luts"].shape).astype(np.uint8)
        _, guard = decode_guarded(to_device(c, cuda_device), n, cuda_device)
        assert np.all(guard == GUARD)


def _quantize_block128(w):
    o, i = w.shape
    t = w.reshape(o // 128, 128, i // 128, 128)
    amax = t.abs().amax(dim=(1, 3), keepdim=True).clamp(min=1e-12)
    return (t * (448.0 / amax)).to(torch.float8_e4m3fn).reshape(o, i)


def test_config1_on_gpu_matches_reference_digests(cuda_device):
    """Config 1 through the GPU packer with the reference's code table: every
    buffer hashes like the reference packer's, and decodes back exactly."""
    from ecf8_b200 import codec
    from ecf8_b200.run import decode_stream
    meta = json.load(open(os.path.join(GOLDEN, "config1_digests.json")))
    w = torch.randn(4096, 4096, generator=torch.Generator().manual_seed(0)) * 0.02
    fp8 = (w * (448.0 / w.abs().max())).to(torch.float8_e4m3fn).flatten().to(cuda_device)
    exps, packed = codec.get_exponents_and_other_4bits_fp8_e4m3(fp8)
    table = {int(a): (int(b), int(c)) for a, b, c in
             zip(meta["table_symbols"], meta["table_bits"], meta["table_values"])}
    table[codec.EOF] = (meta["eof_bits"], meta["eof_value"])
    enc, gaps, op = codec.encode_exponents_for_cuda(exps, codec.HuffmanCode(table))
    luts = codec.get_luts_from_huffman_table(table).to(cuda_device)
    sha = lambda t: hashlib.sha256(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest()
    assert sha(enc) == meta["sha256"]["encoded"]
    assert sha(gaps) == meta["sha256"]["gaps"]
    assert sha(op) == meta["sha256"]["output_positions"]
    assert sha(packed) == meta["sha256"]["packed"]
    out = decode_stream(luts, enc, packed.contiguous(), op, gaps)
    assert torch.equal(out.view(torch.uint8), fp8.view(torch.uint8))


def test_full_qwen3_8b_layer_round_trip(cuda_device):
    """One Qwen3-8B-shaped layer stream (192,937,984 elements, 128x128 block
    scales, sub-Linears in sorted-name order): GPU encode -> decode is the
    identity, and a second decode into the same scratch gives the same bytes."""
    from ecf8_b200.codec import compress_fp8
    from ecf8_b200.run import decode_stream
    shapes = [("mlp.down_proj", 4096, 12288), ("mlp.gate_proj", 12288, 4096), ("mlp.up_proj", 12288, 4096),
              ("self_attn.k_proj", 1024, 4096), ("self_attn.o_proj", 4096, 4096),
              ("self_attn.q_proj", 4096, 4096), ("self_attn.v_proj", 1024, 4096)]
    g = torch.Generator(device=cuda_device).manual_seed(0)
    flat = torch.cat([_quantize_block128(torch.randn(o, i, generator=g, device=cuda_device) * 0.02).reshape(-1)
                      for _, o, i in shapes])
    assert flat.numel() == 192_937_984
    c = compress_fp8(flat)
    assert 2.4 < c["entropy"] < 2.8
    out = decode_stream(c["luts"], c["encoded"], c["packed_other_4bits"], c["output_positions"], c["gaps"])
    assert torch.equal(out.view(torch.uint8), flat.view(torch.uint8))
    out2 = decode_stream(c["luts"], c["encoded"], c["packed_other_4bits"], c["output_positions"], c["gaps"],
                         out)
    assert torch.equal(out2.view(torch.uint8), flat.view(torch.uint8))


@pytest.mark.parametrize("name", golden_names())
def test_golden_streams_with_prepared_table(cuda_device, name):
    """A table prepared once by ecf8_build_table decodes exactly like the
    table the kernel derives itself."""
    from ecf8_b200.run import build_decode_table, decode_stream
    s = load_golden(name)
    d = to_device(s, cuda_device)
    table = build_decode_table(d["luts"])
    n = s["fp8"].size
    buf = torch.full((n + 64,), GUARD, dtype=torch.uint8, device=cuda_device)
    decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"],
                  buf[32:32 + n], table=table)
    derived, _ = decode_guarded(d, n, cuda_device)
    b = buf.cpu().numpy()
    assert np.all(b[:32] == GUARD) and np.all(b[32 + n:] == GUARD)
    assert np.array_equal(b[32:32 + n], s["fp8"])
    assert np.array_equal(b[32:32 + n], derived)


@pytest.mark.parametrize("seed", range(20))
def test_random_streams_with_prepared_table(cuda_device, oracle_mod, seed):
    from ecf8_b200.run import build_decode_table, decode_stream
    rng = np.random.default_rng(5000 + seed)
    s = random_stream(oracle_mod, rng)
    d = to_device(s, cuda_device)
    out = decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"],
                        table=build_decode_table(d["luts"]))
    assert np.array_equal(out.view(torch.uint8).cpu().numpy(), s["fp8"])


def test_batch_mixing_prepared_and_derived_tables(cuda_device):
    from ecf8_b200.run import build_decode_table, decode_streams
    names = golden_names()
    ss = [load_golden(n) for n in names]
    ds = [to_device(s, cuda_device) for s in ss]
    for i, d in enumerate(ds):
        if i % 2 == 0:
            d["decode_table"] = build_decode_table(d["luts"])
    outs = [torch.zeros(s["fp8"].size, dtype=torch.uint8, device=cuda_device) for s in ss]
    decode_streams(ds, outs)
    torch.cuda.synchronize()
    for n, s, o in zip(names, ss, outs):
        assert np.array_equal(o.cpu().numpy(), s["fp8"]), n


def _skewed_stream(oracle, rng, n):
    """A code table from power-of-two counts (codes of 1 to 16 bits) with
    data drawn uniformly over the same 16 symbols: about a sixth of the codes
    are longer than the 13-bit table, so table steps often end the run loop
    for the two-level LUT, at run ends too."""
    from ecf8_b200 import codec
    from helpers import fp8_from_exponents, table_to_arrays
    cnt = {int(s): 1 << i for i, s in enumerate(rng.permutation(16))}
    table = codec.huffman_code_table(cnt)
    luts = codec.get_luts_from_huffman_table(table).numpy()
    bits, vals, eb, ev = table_to_arrays(table)
    e = rng.integers(0, 16, n).astype(np.uint8)
    enc, gaps, op = oracle.encode(e, bits, vals, eb, ev)
    fp8 = fp8_from_exponents(e, rng)
    _, packed = oracle.split(fp8)
    return {"fp8": fp8, "luts": luts, "encoded": enc, "packed": packed, "gaps": gaps,
            "output_positions": op, "table": table, "max_bits": int(bits.max())}


@pytest.mark.parametrize("seed", range(4))
def test_long_codes_everywhere(cuda_device, oracle_mod, seed):
    from ecf8_b200.run import build_decode_table, decode_stream
    rng = np.random.default_rng(700 + seed)
    s = _skewed_stream(oracle_mod, rng, 200000 + 2 * seed)
    assert s["max_bits"] > 13
    d = to_device(s, cuda_device)
    derived, guard = decode_guarded(d, s["fp8"].size, cuda_device)
    assert np.all(guard == GUARD)
    assert np.array_equal(derived, s["fp8"])
    out = decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"],
                        table=build_decode_table(d["luts"]))
    assert np.array_equal(out.view(torch.uint8).cpu().numpy(), s["fp8"])
    if seed == 0:
        assert np.array_equal(run_reference_kernel(s, cuda_device), s["fp8"])


TAB_LUT_OFF = 8192 * 8 + 8192 * 2  # prepared table: entries, end masks, LUT copy, header
TAB_HDR_OFF = TAB_LUT_OFF + 18 * 256


def test_stale_prepared_table_is_not_used(cuda_device, oracle_mod):
    """A table built from another stream's LUTs (e.g. a cache keyed by a
    reused address) is detected by its LUT copy: the kernel derives the
    right table itself and the decode stays exact."""
    from ecf8_b200.run import build_decode_table, decode_stream
    rng = np.random.default_rng(77)
    a = random_stream(oracle_mod, rng, n=200000, k=12)
    b = random_stream(oracle_mod, rng, n=200000, k=5)
    assert not np.array_equal(a["luts"], b["luts"]) or a["luts"].shape != b["luts"].shape
    da, db = to_device(a, cuda_device), to_device(b, cuda_device)
    stale = build_decode_table(db["luts"])
    out = decode_stream(da["luts"], da["encoded"], da["packed_other_4bits"], da["output_positions"],
                        da["gaps"], table=stale)
    assert np.array_equal(out.view(torch.uint8).cpu().numpy(), a["fp8"])


def test_corrupt_prepared_table_stays_in_bounds(cuda_device):
    """A table ecf8_build_table did not write (random words; random entries
    with in-range bit counts but more symbols than bits; random end masks)
    must not make the kernel stall or touch memory outside its buffers."""
    from ecf8_b200 import _lib
    from ecf8_b200.run import decode_stream
    rng = np.random.default_rng(9)
    s = load_golden("gauss_block128")
    d = to_device(s, cuda_device)
    n = s["fp8"].size
    words = _lib.TABLE_BYTES // 4
    for trial in range(4):
        t = rng.integers(0, 2 ** 32, words, dtype=np.uint64).astype(np.uint32)
        if trial % 2:  # entries: bits 1..13, 1..6 symbols (often more than bits)
            ent = t[:16384].reshape(8192, 2)
            b = rng.integers(1, 14, 8192).astype(np.uint32)
            c = rng.integers(1, 7, 8192).astype(np.uint32)
            ent[:, 0] = (ent[:, 0] & 0xffffff00) | b
            ent[:, 1] = (b << 23) | (4 * c)
        # A matching LUT copy and header, so the kernel takes the entries as they are.
        tb = t.view(np.uint8)
        tb[TAB_LUT_OFF:TAB_LUT_OFF + 18 * 256] = 0
        tb[TAB_LUT_OFF:TAB_LUT_OFF + s["luts"].size] = s["luts"].reshape(-1)
        tb[TAB_HDR_OFF:TAB_HDR_OFF + 8] = np.array([0x38464345, s["luts"].shape[0]], np.uint32).view(np.uint8)
        table = torch.from_numpy(t.view(np.int32).copy()).to(cuda_device)
        buf = torch.full((n + 64,), GUARD, dtype=torch.uint8, device=cuda_device)
        decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"],
                      buf[32:32 + n], table=table)
        torch.cuda.synchronize()
        b = buf.cpu().numpy()
        assert np.all(b[:32] == GUARD) and np.all(b[32 + n:] == GUARD)


def test_overlap_previous_back_to_back(cuda_device):
    """ECF8_DECODE_OVERLAP_PREVIOUS: decodes that may start while the previous
    kernel runs, one after another into one buffer (the hook's shared
    scratch), each right after a kernel that writes that buffer, give the same
    bytes as plain decodes; with and without prepared tables."""
    from ecf8_b200.run import build_decode_table, decode_stream
    names = golden_names()
    ss = [load_golden(n) for n in names]
    ds = [to_device(s, cuda_device) for s in ss]
    tables = [build_decode_table(d["luts"]) for d in ds]
    torch.cuda.synchronize()
    n_max = max(s["fp8"].size for s in ss)
    buf = torch.full((n_max + 64,), GUARD, dtype=torch.uint8, device=cuda_device)
    for rep in range(2):
        for s, d, t in zip(ss, ds, tables):
            n = s["fp8"].size
            out = buf[32:32 + n]
            out.fill_(0x5A)  # the previous kernel writes the output region
            decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"],
                          out, table=t if rep == 0 else None, overlap_previous=True)
            b = buf.cpu().numpy()
            assert np.array_equal(b[32:32 + n], s["fp8"])
            assert np.all(b[:32] == GUARD) and np.all(b[32 + n_max:] == GUARD)


def test_overlap_previous_batched_matches_plain(cuda_device):
    from ecf8_b200.run import build_decode_table, decode_streams
    ss = [load_golden(n) for n in golden_names()]
    ds = [to_device(s, cuda_device) for s in ss]
    for d in ds:
        d["decode_table"] = build_decode_table(d["luts"])
    torch.cuda.synchronize()
    for _ in range(3):
        outs = [torch.zeros(s["fp8"].size, dtype=torch.uint8, device=cuda_device) for s in ss]
        decode_streams(ds, outs, overlap_previous=True)
        decode_streams(ds, outs, overlap_previous=True)
        torch.cuda.synchronize()
        for s, o in zip(ss, outs):
            assert np.array_equal(o.cpu().numpy(), s["fp8"])


def test_overlap_previous_waits_for_a_long_kernel_writing_the_outputs(cuda_device):
    """The overlapped decode must not write before the previous kernel has
    completed.  The previous kernel here is a long decode (64 M elements, tens
    of microseconds) of another stream into a buffer that contains the
    overlapped decode's output region; if the second decode wrote early, the
    first would overwrite part of its bytes."""
    from ecf8_b200.codec import compress_fp8
    from ecf8_b200.run import build_decode_table, decode_stream
    g = torch.Generator(device=cuda_device).manual_seed(4)
    n_big = 64 << 20
    big = (torch.randn(n_big, generator=g, device=cuda_device) * 20).to(torch.float8_e4m3fn)
    c = compress_fp8(big)
    tb = build_decode_table(c["luts"])
    buf = torch.empty(n_big, dtype=torch.uint8, device=cuda_device)
    for i, name in enumerate(golden_names()):
        s = load_golden(name)
        d = to_device(s, cuda_device)
        t = build_decode_table(d["luts"])
        n = s["fp8"].size
        off = (n_big - n) // 2 if i % 2 else n_big - n - 16 * i
        torch.cuda.synchronize()
        decode_stream(c["luts"], c["encoded"], c["packed_other_4bits"], c["output_positions"], c["gaps"], buf,
                      table=tb)
        decode_stream(d["luts"], d["encoded"], d["packed_other_4bits"], d["output_positions"], d["gaps"],
                      buf[off:off + n], table=t, overlap_previous=True)
        torch.cuda.synchronize()
        assert np.array_equal(buf[off:off + n].cpu().numpy(), s["fp8"]), name
        ref = big.view(torch.uint8)
        assert torch.equal(buf[:off], ref[:off]) and torch.equal(buf[off + n:], ref[off + n:])
