"""``dfloat.utils`` names (dfloat/utils.py of the reference): the codec that
writes the ECF8 stream format and the model-walk helpers, from ecf8_b200."""

from ecf8_b200.codec import (  # noqa: F401
    compute_shannon_entropy,
    encode_exponents_for_cuda,
    find_layers_by_data_type,
    find_layers_by_data_type_and_layer_type,
    find_layers_by_layer_type,
    find_layers_by_selection,
    flatten_block_of_weights,
    get_exponents_and_other_4bits_fp8_e4m3,
    get_luts_from_huffman_table,
    get_nbit_codec,
    locate_block_by_regex,
    repo_id_to_model_id,
)
from ecf8_b200.run import param_to_bytes, report_model_size  # noqa: F401
