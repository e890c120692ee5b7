"""ecf8_b200: B200-native (sm_100a) ECF8 decode engine.

Drop-in for the decode path of zeyuyang8/ecf8's ``dfloat`` package: the names
below are those of ``dfloat.run`` (dfloat/run/__init__.py:1-17) plus the
codec functions of ``dfloat.utils`` that produce the stream format.  The decode
kernels live in libecf8_b200.so (C ABI: include/ecf8.h).
"""

from .codec import (  # noqa: F401
    compress_fp8,
    compute_shannon_entropy,
    encode_exponents_for_cuda,
    flatten_block_of_weights,
    get_exponents_and_other_4bits_fp8_e4m3,
    get_luts_from_huffman_table,
    get_nbit_codec,
)
from .run import (  # noqa: F401
    DFloatDiffSynthModelFP8,
    DFloatModel,
    HostStreamDecoder,
    TensorManager,
    _decode,
    build_decode_table,
    decode_stream,
    decode_streams,
    enable_decode_prefetch,
    get_dfloat_model_name_or_path,
    get_hook,
    load_and_replace_tensors,
    load_and_replace_tensors_parallel,
)

__version__ = "0.1.0"

__all__ = [
    "DFloatModel",
    "_decode",
    "get_dfloat_model_name_or_path",
    "load_and_replace_tensors",
    "load_and_replace_tensors_parallel",
    "DFloatDiffSynthModelFP8",
]
