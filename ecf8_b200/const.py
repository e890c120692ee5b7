"""Which blocks of a model family are ECF8 streams.

The block patterns are part of the compressed-checkpoint contract: a
checkpoint's pattern_dict.json is written from them and the loader matches
module names against them, so they must equal the reference's tables
(dfloat/const.py:1-151) for the families kept here.  A list value means the
whole matched block is one stream; a dict value maps a block pattern to the
sub-Linear names (in sorted order) that are concatenated into its stream.
"""

FP8_PATTERN_DICT = {
    "llm": {
        "bf16": [r"model\.embed_tokens", r"lm_head"],
        "fp8": [r"model\.layers\.\d+"],
    },
    "deepseekv3": {
        "bf16": [r"model\.embed_tokens", r"lm_head"],
        "fp8": [
            r"model\.layers\.[0-2]",
            r"model\.layers\.(?![0-2](?:[^0-9]|$))\d+\.self_attn",
            r"model\.layers\.(?![0-2](?:[^0-9]|$))\d+\.mlp\.shared_experts",
            r"model\.layers\.(?![0-2](?:[^0-9]|$))\d+\.mlp\.experts\.\d+",
        ],
    },
    "qwen3moe": {
        "bf16": [r"model\.embed_tokens", r"lm_head"],
        "fp8": [r"model\.layers\.\d+\.self_attn", r"model\.layers\.\d+\.mlp\.experts\.\d+"],
    },
    "diffsynth-flux-fp8": {
        "fp8": {
            r"text_encoder_2\.encoder\.block\.\d+": [
                "layer.0.SelfAttention.k", "layer.0.SelfAttention.o",
                "layer.0.SelfAttention.q", "layer.0.SelfAttention.v",
            ],
            r"dit\.blocks\.\d+": [
                "attn.a_to_out", "attn.a_to_qkv", "attn.b_to_out", "attn.b_to_qkv",
                "ff_a.0", "ff_a.2", "ff_b.0", "ff_b.2",
            ],
            r"dit\.single_blocks\.\d+": ["norm.linear", "proj_out", "to_qkv_mlp"],
        },
        "bf16": [],
    },
}

MODEL_CLASS_MAP = {
    "llm": {"Qwen3ForCausalLM", "LlamaForCausalLM"},
    "deepseekv3": {"DeepseekV3ForCausalLM"},
    "qwen3moe": {"Qwen3MoeForCausalLM"},
    # FluxDiTPipeline: the FLUX-shaped DiT of ecf8_b200.dit_model (same block names)
    "diffsynth-flux-fp8": {"FluxImagePipeline", "FluxDiTPipeline"},
}

DEFAULT_NO_SPLIT_PATTERN = {
    "llm": [r"model\.embed_tokens", r"model\.layers\.\d+", r"lm_head"],
    "deepseekv3": [r"model\.embed_tokens", r"model\.layers\.\d+", r"lm_head"],
    "qwen3moe": [r"model\.embed_tokens", r"model\.layers\.\d+", r"lm_head"],
    "diffsynth-flux-fp8": [
        r"text_encoder_2\.encoder\.block\.\d+", r"dit\.blocks\.\d+", r"dit\.single_blocks\.\d+",
    ],
}


def _family(model_class):
    for key, classes in MODEL_CLASS_MAP.items():
        if model_class in classes:
            return key
    raise ValueError(f"Model class {model_class} not supported")


def get_fp8_pattern_dict(model_class):
    return FP8_PATTERN_DICT[_family(model_class)]


def get_default_no_split_pattern(model_class):
    return DEFAULT_NO_SPLIT_PATTERN[_family(model_class)]
