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
