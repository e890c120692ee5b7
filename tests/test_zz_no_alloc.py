"""ecf8_encode_noalloc: the packer for callers that cannot allocate.

Some callers cannot give the library extra device memory: a host framework
that owns all device memory through its own pool (an out-of-band cudaMalloc
can fail there or fragment the pool), or a checkpoint loader that must not
trigger cudaMalloc's implicit device synchronisation while other streams run.
For them ecf8_encode_noalloc packs a stream in one call, with its working
memory built into the library.  These tests call it through the C ABI twice
in a row (a long stream, then a shorter one, so stale scratch from the first
call would show) and require the exact bytes of the workspace-based packer
(ecf8_encode_plan / ecf8_encode_emit).  This file is collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import random_stream

pytestmark = pytest.mark.gpu


def noalloc_pack(exps, table, dev):
    """Packs with ecf8_encode_noalloc; returns (encoded, gaps, output_positions)
    cut to the sizes the call reports."""
    from ecf8_b200 import _lib
    from ecf8_b200.codec import EOF
    L = _lib.lib()
    bits = np.zeros(16, np.uint8)
    vals = (ctypes.c_uint32 * 16)()
    for s, (b, v) in table.items():
        if isinstance(s, int):
            bits[s], vals[s] = b, v
    eb, ev = table[EOF]
    n = exps.numel()
    max_bytes = -(-n * int(bits.max()) // 8)
    groups = -(-max_bytes // 4096)
    enc = torch.empty((max_bytes + 3) & ~3, dtype=torch.uint8, device=dev)
    gaps = torch.empty(max(groups * 256, 4), dtype=torch.uint8, device=dev)
    op = torch.empty(groups + 2, dtype=torch.int64, device=dev)
    sizes = torch.empty(3, dtype=torch.int64, device=dev)
    st = L.ecf8_encode_noalloc(exps.data_ptr(), n, bits.tobytes(), vals, eb, ev, enc.data_ptr(), enc.numel(),
                               gaps.data_ptr(), gaps.numel(), op.data_ptr(), op.numel(), sizes.data_ptr(),
                               torch.cuda.current_stream(dev).cuda_stream)
    assert st == 0, L.ecf8_status_string(st)
    return enc, gaps, op, sizes


def test_noalloc_packer_matches_workspace_packer_twice_in_a_row(cuda_device, oracle_mod):
    from ecf8_b200.codec import HuffmanCode, encode_exponents_for_cuda
    from ecf8_b200.run import decode_stream
    rng = np.random.default_rng(77)
    streams = [random_stream(oracle_mod, rng, n=900_000, k=16, alpha=5.0),
               random_stream(oracle_mod, rng, n=70_000, k=9, alpha=0.3)]
    exps = [torch.from_numpy(((s["fp8"] >> 3) & 15).astype(np.uint8)).to(cuda_device) for s in streams]
    want = [encode_exponents_for_cuda(e, HuffmanCode(s["table"])) for e, s in zip(exps, streams)]
    got = [noalloc_pack(e, s["table"], cuda_device) for e, s in zip(exps, streams)]  # two calls in a row
    torch.cuda.synchronize()
    for s, (we, wg, wo), (ge, gg, go, sz) in zip(streams, want, got):
        total_bits, n_bytes, n_op = sz.cpu().tolist()
        assert n_bytes == we.numel() and n_op == wo.numel()
        assert torch.equal(ge[:n_bytes], we)
        assert torch.equal(gg[:wg.numel()], wg)
        assert not gg[wg.numel():].any()
        assert torch.equal(go[:n_op], wo.view(torch.int64))
        assert np.array_equal(ge[:n_bytes].cpu().numpy(), s["encoded"])  # and the oracle packer's bytes
        out = decode_stream(torch.from_numpy(s["luts"]).to(cuda_device), ge[:n_bytes].contiguous(),
                            torch.from_numpy(s["packed"]).to(cuda_device), go[:n_op].contiguous(),
                            gg[:wg.numel()].contiguous())
        assert np.array_equal(out.view(torch.uint8).cpu().numpy(), s["fp8"])


def test_noalloc_packer_rejects_streams_beyond_its_scratch(cuda_device):
    from ecf8_b200 import _lib
    L = _lib.lib()
    bits = bytes([2] * 16)
    vals = (ctypes.c_uint32 * 16)(*([0, 1, 2, 3] * 4))
    n = _lib.NOALLOC_MAX_ELEMENTS + 2
    # Rejected on the host before any device work: the pointers are never used.
    st = L.ecf8_encode_noalloc(16, n, bits, vals, 2, 3, 16, 1 << 40, 16, 1 << 40, 16, 1 << 30, 16, None)
    assert st == _lib.ERR_TOO_LARGE
    assert b"268,435,456" in L.ecf8_status_string(st)


def test_noalloc_packer_rejects_invalid_exponents_on_the_device(cuda_device):
    """Exponent bytes above 15 (or symbols without a code) are found on the
    device: sizes come back {0, 0, 0}, the outputs stay cleared and nothing
    outside them is written.  A valid call right after works as before."""
    from ecf8_b200 import _lib
    L = _lib.lib()
    rng = np.random.default_rng(8)
    bits = np.zeros(16, np.uint8)
    bits[:4] = [1, 2, 3, 3]
    vals = (ctypes.c_uint32 * 16)(*([0, 2, 6, 7] + [0] * 12))
    e = torch.from_numpy(rng.integers(0, 4, 20000).astype(np.uint8)).to(cuda_device)
    e[123] = 77
    n = e.numel()
    max_bytes = -(-n * 3 // 8)
    groups = -(-max_bytes // 4096)
    guard = 64
    enc = torch.full((((max_bytes + 3) & ~3) + 2 * guard,), 0xA5, dtype=torch.uint8, device=cuda_device)
    gaps = torch.full((groups * 256 + 2 * guard,), 0xA5, dtype=torch.uint8, device=cuda_device)
    op = torch.full((groups + 2 + 16,), -1, dtype=torch.int64, device=cuda_device)
    sizes = torch.full((3,), -1, dtype=torch.int64, device=cuda_device)
    st = torch.cuda.current_stream(cuda_device).cuda_stream
    r = L.ecf8_encode_noalloc(e.data_ptr(), n, bits.tobytes(), vals, 4, 15, enc[guard:].data_ptr(),
                              enc.numel() - 2 * guard, gaps[guard:].data_ptr(), gaps.numel() - 2 * guard,
                              op[8:].data_ptr(), groups + 2, sizes.data_ptr(), st)
    assert r == 0
    torch.cuda.synchronize()
    assert sizes.cpu().tolist() == [0, 0, 0]
    assert not enc[guard:-guard].any() and torch.all(enc[:guard] == 0xA5) and torch.all(enc[-guard:] == 0xA5)
    assert not gaps[guard:-guard].any() and torch.all(gaps[:guard] == 0xA5) and torch.all(gaps[-guard:] == 0xA5)
    assert not op[8:8 + groups + 2].any() and torch.all(op[:8] == -1) and torch.all(op[8 + groups + 2:] == -1)
    e[123] = 1
    table = {s: (int(bits[s]), int(vals[s])) for s in range(4)}
    from ecf8_b200.codec import EOF
    table[EOF] = (4, 15)
    got = noalloc_pack(e, table, cuda_device)
    torch.cuda.synchronize()
    assert got[3].cpu().tolist()[1] > 0
