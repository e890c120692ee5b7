"""Generation harness (config 3) on a shortened model: the compressed arm,
decoding every layer in its forward-pre-hook, generates the same tokens with
bit-identical logits as the uncompressed FP8 model."""
import pytest

pytestmark = pytest.mark.gpu


def test_generation_identical_logits(cuda_device):
    from ecf8_b200.inference_llm import main
    line = main(["--synthetic", "--num_layers", "2", "--batch_size", "2", "--prompt_len", "16",
                 "--num_tokens", "8", "--keep", "8"])
    assert line["identical_tokens"] and line["identical_logit_sums_all_steps"]
    assert line["identical_full_logits_first_steps"]
    assert line["compressed"]["new_tokens"] == 8 == line["uncompressed"]["new_tokens"]
    assert 0 < line["ecf8_stream_bytes"] < line["fp8_weight_bytes"]
