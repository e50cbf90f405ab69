"""graphkv_b200 -- B200-native (sm_100a) GraphKV KV-cache compression.

Drop-in for the reference package's compression path: ``quantize_hf_cache``,
``QuantizedKvCache`` (``stats()``, ``dequantize()``, ``to_hf_cache()``),
``KvQuantConfig`` and the named profiles.  Compute runs in the CUDA kernels of
``graphkv_b200/lib/libgraphkv_b200.so``; there is no CPU fallback.
"""
from .config import KvQuantConfig
from .core import (
    QuantizedKvCache,
    QuantizedKvLayer,
    QuantizedTensor,
    attention_from_kv,
    attention_from_quantized,
    attention_report,
    build_retention_mask,
    chunk_scores_to_token_scores,
    hf_cache_to_tuple,
    quantize_kv_layer,
)
from .graph_model import (
    GraphFactBank,
    GraphMemory17L,
    GraphMemoryConfig,
    GraphMemoryRequest,
    GraphMnemeRequest,
    GraphQueryBank,
    GraphRetentionChunk,
    build_candidate_bank,
    build_fact_bank,
    build_graph_mneme_token_scores,
    build_query_bank,
    bundled_graph_model_dir,
    bundled_graph_model_metadata,
    graph_mneme_chunk_scores,
    graph_mneme_request_token_scores,
    graph_mneme_token_scores,
    load_bundled_graph_model,
    normalize_graph_scores,
)
from .integrations import (
    llama_cpp_args,
    llama_cpp_command,
    llama_cpp_env,
    quantize_hf_cache,
    vllm_cli_args,
    vllm_kwargs,
)
from .profiles import GraphKVProfile, get_profile, list_profiles

__version__ = "0.1.0"

__all__ = [
    "GraphFactBank",
    "GraphKVProfile",
    "GraphMemory17L",
    "GraphMemoryConfig",
    "GraphMemoryRequest",
    "GraphMnemeRequest",
    "GraphQueryBank",
    "GraphRetentionChunk",
    "KvQuantConfig",
    "QuantizedKvCache",
    "QuantizedKvLayer",
    "QuantizedTensor",
    "attention_from_kv",
    "attention_from_quantized",
    "attention_report",
    "build_candidate_bank",
    "build_fact_bank",
    "build_graph_mneme_token_scores",
    "build_query_bank",
    "build_retention_mask",
    "bundled_graph_model_dir",
    "bundled_graph_model_metadata",
    "chunk_scores_to_token_scores",
    "get_profile",
    "graph_mneme_chunk_scores",
    "graph_mneme_request_token_scores",
    "graph_mneme_token_scores",
    "hf_cache_to_tuple",
    "list_profiles",
    "llama_cpp_args",
    "llama_cpp_command",
    "llama_cpp_env",
    "load_bundled_graph_model",
    "normalize_graph_scores",
    "quantize_hf_cache",
    "quantize_kv_layer",
    "vllm_cli_args",
    "vllm_kwargs",
]
