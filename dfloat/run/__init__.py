"""``dfloat.run`` names (dfloat/run/__init__.py:1-17 of the reference)."""

from .run import (  # noqa: F401
    DFloatDiffSynthModelFP8,
    DFloatModel,
    _decode,
    get_dfloat_model_name_or_path,
    load_and_replace_tensors,
    load_and_replace_tensors_parallel,
)

__all__ = [
    "DFloatModel",
    "_decode",
    "get_dfloat_model_name_or_path",
    "load_and_replace_tensors",
    "load_and_replace_tensors_parallel",
    "DFloatDiffSynthModelFP8",
]
