"""Expert-parallel MoE harness on one GPU (test-sized): with its attention
blocks and experts compressed (experts decoded in one batched launch when
routed) the model generates identical tokens and logits."""
import pytest

pytestmark = pytest.mark.gpu


def test_compressed_moe_generation_identical(cuda_device):
    from ecf8_b200.inference_moe import main
    line = main(["--small", "--layers", "2", "--batch", "2", "--prompt_len", "8", "--new_tokens", "6"])
    assert line["identical_tokens_all_ranks"] and line["identical_logit_sums_all_ranks"]
    assert 0 < line["ecf8_stream_bytes_per_rank"]
