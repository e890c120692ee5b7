"""DiT denoising harness (config 4) on a shortened model: the compressed arm
gives bit-identical latents and velocities."""
import pytest

pytestmark = pytest.mark.gpu


def test_dit_denoising_identical(cuda_device):
    from ecf8_b200.inference_dit import main
    line = main(["--n_double", "1", "--n_single", "2", "--image_tokens", "256", "--text_tokens", "64",
                 "--steps", "3", "--warm", "1"])
    assert line["finite_output"]
    assert line["identical_latents"] and line["identical_velocity_sums_all_steps"]
    assert 0 < line["ecf8_stream_bytes"] < line["fp8_weights"]
