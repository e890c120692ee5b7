"""The FP8 Linear both end-to-end arms share: the block-scaled FP8 GEMM that
reads e4m3 weights directly agrees with the bf16 expansion of the same
weights (within FP8 activation rounding) and is deterministic, so identical
decoded weights give identical outputs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_block_scaled_fp8_gemm_matches_expansion_and_is_deterministic(cuda_device):
    from ecf8_b200 import fp8_model
    lin = fp8_model.Fp8Linear(4096, 12288, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(0)
    q, s = fp8_model.quantize_block128(torch.randn(12288, 4096, generator=g, device=cuda_device) * 0.02)
    lin.weight.data.copy_(q)
    lin.weight_scale_inv.copy_(s)
    backend = fp8_model.fp8_matmul_backend()
    for m in (16, 2048):
        x = torch.randn(m, 4096, generator=g, device=cuda_device).to(torch.bfloat16)
        y = lin(x)
        ref = torch.nn.functional.linear(x.float(), lin.dequantized(torch.float32))
        rel = ((y.float() - ref).norm() / ref.norm()).item()
        assert rel < 0.05, (backend, m, rel)  # e4m3 activations: ~2-3 % relative error
        assert torch.equal(lin(x), y)
    # a view of another buffer (how the decode hook injects weights) gives the same bytes
    buf = torch.empty(q.numel() + 256, dtype=torch.float8_e4m3fn, device=cuda_device)
    buf[128:128 + q.numel()] = q.reshape(-1)
    lin2 = fp8_model.Fp8Linear(4096, 12288, device=cuda_device)
    lin2.weight_scale_inv.copy_(s)
    del lin2.weight
    lin2.weight = buf[128:128 + q.numel()].view(12288, 4096)
    assert torch.equal(lin2(x), lin(x))
    print("fp8 matmul backend:", backend)
