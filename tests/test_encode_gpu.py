"""GPU packer parity: byte-identical to the reference packer (golden streams)
and to its oracle restatement (random streams)."""
import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from helpers import random_stream

pytestmark = pytest.mark.gpu


def codec_from(table_symbols, table_bits, table_values, eof_bits, eof_value):
    from ecf8_b200 import codec
    t = {int(a): (int(b), int(c)) for a, b, c in zip(table_symbols, table_bits, table_values)}
    t[codec.EOF] = (int(eof_bits), int(eof_value))
    return codec.HuffmanCode(t)


@pytest.mark.parametrize("name", golden_names())
def test_gpu_packer_matches_reference_packer(cuda_device, name):
    from ecf8_b200.codec import encode_exponents_for_cuda
    s = load_golden(name)
    exps = torch.from_numpy(((s["fp8"] >> 3) & 15).astype(np.uint8)).to(cuda_device)
    c = codec_from(s["table_symbols"], s["table_bits"], s["table_values"], s["eof_bits"], s["eof_value"])
    enc, gaps, op = encode_exponents_for_cuda(exps, c)
    assert np.array_equal(enc.cpu().numpy(), s["encoded"])
    assert np.array_equal(gaps.cpu().numpy(), s["gaps"])
    assert np.array_equal(op.view(torch.int64).cpu().numpy().view(np.uint64), s["output_positions"])


@pytest.mark.parametrize("seed", range(20))
def test_gpu_packer_matches_oracle_on_random_streams(cuda_device, oracle_mod, seed):
    from ecf8_b200.codec import HuffmanCode, encode_exponents_for_cuda
    rng = np.random.default_rng(50 + seed)
    s = random_stream(oracle_mod, rng, n=int(rng.integers(1, 400000)) * 2)
    exps = torch.from_numpy(((s["fp8"] >> 3) & 15).astype(np.uint8)).to(cuda_device)
    enc, gaps, op = encode_exponents_for_cuda(exps, HuffmanCode(s["table"]))
    assert np.array_equal(enc.cpu().numpy(), s["encoded"])
    assert np.array_equal(gaps.cpu().numpy(), s["gaps"])
    assert np.array_equal(op.view(torch.int64).cpu().numpy().view(np.uint64), s["output_positions"])


def test_cpu_input_round_trips_to_cpu(cuda_device):
    from ecf8_b200.codec import encode_exponents_for_cuda
    s = load_golden("tiny_130")
    exps = torch.from_numpy(((s["fp8"] >> 3) & 15).astype(np.uint8))
    c = codec_from(s["table_symbols"], s["table_bits"], s["table_values"], s["eof_bits"], s["eof_value"])
    enc, gaps, op = encode_exponents_for_cuda(exps, c)
    assert enc.device.type == "cpu" and op.dtype == torch.uint64
    assert np.array_equal(enc.numpy(), s["encoded"])


def _plan_emit_raw(exps, bits, vals, eb, ev, dev):
    """ecf8_encode_plan + ecf8_encode_emit through the C ABI, outputs inside
    guard-filled buffers; returns (plan = [invalid exponents, total bits,
    encoded bytes, output positions], encoded, gaps, op) with the guards."""
    import ctypes
    from ecf8_b200 import _lib
    L = _lib.lib()
    n = exps.numel()
    st = torch.cuda.current_stream(dev).cuda_stream
    ws = torch.zeros(L.ecf8_encode_workspace_bytes(n), dtype=torch.uint8, device=dev)
    assert L.ecf8_encode_plan(exps.data_ptr(), n, bits.tobytes(), eb, ws.data_ptr(), st) == 0
    plan = ws[-32:].view(torch.int64).cpu().tolist()
    cap = 4096 * 4
    enc = torch.full((cap + 64,), 0xA5, dtype=torch.uint8, device=dev)
    gaps = torch.full((4 * 256 + 64,), 0xA5, dtype=torch.uint8, device=dev)
    op = torch.full((16,), -1, dtype=torch.int64, device=dev)
    cv = (ctypes.c_uint32 * 16)(*[int(x) for x in vals])
    n_bytes, n_op = plan[2], max(plan[3], 1)
    assert 0 < n_bytes <= cap and n_op <= 8
    n_gap = -(-n_bytes // 4096) * 256
    assert L.ecf8_encode_emit(exps.data_ptr(), n, bits.tobytes(), cv, eb, ev, ws.data_ptr(), enc[32:].data_ptr(),
                              n_bytes, cap, gaps[32:].data_ptr(), n_gap, op[4:].data_ptr(), n_op, st) == 0
    torch.cuda.synchronize()
    return plan, enc, gaps, op


def test_invalid_exponents_are_counted_and_nothing_is_emitted(cuda_device):
    """Exponent bytes above 15 and symbols without a code: the plan counts
    them, emit writes nothing past the cleared outputs, and nothing outside
    the buffers (the guard bytes stay)."""
    from ecf8_b200.codec import HuffmanCode, encode_exponents_for_cuda
    rng = np.random.default_rng(5)
    bits = np.zeros(16, np.uint8)
    vals = np.zeros(16, np.uint32)
    bits[:4], vals[:4] = [1, 2, 3, 3], [0, 2, 6, 7]
    good = torch.from_numpy(rng.integers(0, 4, 5000).astype(np.uint8)).to(cuda_device)
    for bad_value, n_bad in ((200, 3), (9, 5), (16, 1)):  # above 15 / a symbol without a code
        e = good.clone()
        e[torch.from_numpy(rng.choice(e.numel(), n_bad, replace=False)).to(cuda_device)] = bad_value
        plan, enc, gaps, op = _plan_emit_raw(e, bits, vals, 4, 15, cuda_device)
        assert plan[0] == n_bad
        assert torch.all(enc[:32] == 0xA5) and torch.all(enc[32 + 4096 * 4:] == 0xA5)
        assert not enc[32:32 + 4096 * 4].any()
        assert torch.all(gaps[:32] == 0xA5)
        assert torch.all(op[:4] == -1) and torch.all(op[12:] == -1)
    table = {s: (int(bits[s]), int(vals[s])) for s in range(4)}
    from ecf8_b200.codec import EOF
    table[EOF] = (4, 15)
    e = good.clone()
    e[7] = 200
    with pytest.raises(ValueError):
        encode_exponents_for_cuda(e, HuffmanCode(table))
    plan, enc, _, _ = _plan_emit_raw(good, bits, vals, 4, 15, cuda_device)
    assert plan[0] == 0 and enc[32:32 + plan[2]].any()
