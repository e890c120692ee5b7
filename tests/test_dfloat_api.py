"""The reference's ``dfloat`` import path resolves to this engine: the public
names of dfloat/run/__init__.py:1-17, dfloat/run/run.py, dfloat/utils.py and
dfloat/const.py import unchanged and are the ecf8_b200 objects."""
import importlib

import pytest

RUN_ALL = ["DFloatModel", "_decode", "get_dfloat_model_name_or_path", "load_and_replace_tensors",
           "load_and_replace_tensors_parallel", "DFloatDiffSynthModelFP8"]
RUN_MODULE = RUN_ALL + ["TensorManager", "get_hook", "get_no_split_classes", "_process_compressed_tensor"]
UTILS = ["param_to_bytes", "report_model_size", "repo_id_to_model_id", "locate_block_by_regex",
         "find_layers_by_selection", "find_layers_by_layer_type", "find_layers_by_data_type",
         "find_layers_by_data_type_and_layer_type", "flatten_block_of_weights",
         "get_exponents_and_other_4bits_fp8_e4m3", "compute_shannon_entropy", "get_nbit_codec",
         "get_luts_from_huffman_table", "encode_exponents_for_cuda"]
CONST = ["FP8_PATTERN_DICT", "MODEL_CLASS_MAP", "DEFAULT_NO_SPLIT_PATTERN", "get_fp8_pattern_dict",
         "get_default_no_split_pattern"]


def test_dfloat_run_exports_the_reference_names():
    import dfloat
    import dfloat.run as run
    import ecf8_b200.run as impl
    assert dfloat.__version__
    assert sorted(run.__all__) == sorted(RUN_ALL)
    for name in RUN_ALL:
        assert getattr(run, name) is getattr(impl, name)


@pytest.mark.parametrize("module,names", [("dfloat.run.run", RUN_MODULE), ("dfloat.utils", UTILS),
                                          ("dfloat.const", CONST)])
def test_dfloat_modules_export_the_reference_names(module, names):
    m = importlib.import_module(module)
    for name in names:
        assert hasattr(m, name), f"{module}.{name}"


def test_dfloat_const_matches_the_checkpoint_contract():
    from dfloat.const import get_default_no_split_pattern, get_fp8_pattern_dict
    assert get_fp8_pattern_dict("Qwen3ForCausalLM")["fp8"] == [r"model\.layers\.\d+"]
    assert get_default_no_split_pattern("Qwen3ForCausalLM")


def test_get_no_split_classes():
    import torch.nn as nn
    from dfloat.run.run import get_no_split_classes
    m = nn.Sequential(nn.Linear(2, 2), nn.Sequential(nn.ReLU(), nn.Linear(2, 2)))
    assert get_no_split_classes(m, [r"\d+"]) == ["Linear", "Sequential"]
