"""Public names and engine recipes of the package (reference
``src/graphkv/__init__.py:45-82``, ``src/graphkv/integrations.py:65-124``)."""
import pytest

import graphkv_b200 as gkv

REFERENCE_ALL = {
    "GraphKVProfile", "GraphFactBank", "GraphMemory17L", "GraphMemoryConfig", "GraphMemoryRequest",
    "GraphMnemeRequest", "GraphQueryBank", "GraphRetentionChunk", "KvQuantConfig", "QuantizedKvCache",
    "QuantizedKvLayer", "attention_from_kv", "attention_report", "build_retention_mask", "build_candidate_bank",
    "build_fact_bank", "build_graph_mneme_token_scores", "build_query_bank", "bundled_graph_model_metadata",
    "bundled_graph_model_dir", "chunk_scores_to_token_scores", "get_profile", "graph_mneme_chunk_scores",
    "graph_mneme_request_token_scores", "graph_mneme_token_scores", "hf_cache_to_tuple", "list_profiles",
    "load_bundled_graph_model", "llama_cpp_args", "llama_cpp_command", "llama_cpp_env", "normalize_graph_scores",
    "quantize_hf_cache", "quantize_kv_layer", "vllm_cli_args", "vllm_kwargs",
}


def test_every_reference_name_is_exported():
    assert REFERENCE_ALL <= set(gkv.__all__)
    for name in gkv.__all__:
        assert hasattr(gkv, name), name
    assert gkv.GraphMnemeRequest is gkv.GraphMemoryRequest


def test_vllm_recipes():
    assert gkv.vllm_kwargs() == {"kv_cache_dtype": "fp8", "calculate_kv_scales": True}
    assert gkv.vllm_kwargs("vllm-fp8", max_model_len=4096) == {"kv_cache_dtype": "fp8", "calculate_kv_scales": False,
                                                               "max_model_len": 4096}
    assert gkv.vllm_cli_args() == ["--kv-cache-dtype", "fp8", "--calculate-kv-scales"]
    assert gkv.vllm_cli_args("vllm-fp8") == ["--kv-cache-dtype", "fp8"]
    with pytest.raises(ValueError, match="is not a vLLM profile"):
        gkv.vllm_kwargs("graphkv")


def test_llama_cpp_recipes():
    assert gkv.llama_cpp_args() == ["--cache-type-k", "q8_0", "--cache-type-v", "q8_0"]
    assert gkv.llama_cpp_env("llamacpp-q4") == {"LLAMA_ARG_CACHE_TYPE_K": "q4_0", "LLAMA_ARG_CACHE_TYPE_V": "q4_0"}
    assert gkv.llama_cpp_command("my model.gguf", extra_args=["-n", "16"]) == \
        "llama-cli -m 'my model.gguf' --cache-type-k q8_0 --cache-type-v q8_0 -n 16"
    with pytest.raises(ValueError, match="is not a llama.cpp profile"):
        gkv.llama_cpp_args("vllm-fp8")


def test_engine_profiles_are_rejected_by_quantize_hf_cache():
    with pytest.raises(ValueError, match="engine-native recipe"):
        gkv.quantize_hf_cache(((None, None),), "vllm-fp8")
