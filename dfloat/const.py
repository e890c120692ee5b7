"""``dfloat.const`` names (dfloat/const.py of the reference): the pattern
tables compressed checkpoints record, from ecf8_b200.const."""

from ecf8_b200.const import (  # noqa: F401
    DEFAULT_NO_SPLIT_PATTERN,
    FP8_PATTERN_DICT,
    MODEL_CLASS_MAP,
    get_default_no_split_pattern,
    get_fp8_pattern_dict,
)
