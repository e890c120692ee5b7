"""``dfloat.run.run`` names (dfloat/run/run.py of the reference): scratch,
hook, kernel launcher, loaders and model wrappers of ecf8_b200.run."""

from ecf8_b200.run import (  # noqa: F401
    DFloatDiffSynthModelFP8,
    DFloatModel,
    TensorManager,
    _decode,
    _process_compressed_tensor,
    get_dfloat_model_name_or_path,
    get_hook,
    get_no_split_classes,
    load_and_replace_tensors,
    load_and_replace_tensors_parallel,
)
