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
    attention_report,
    build_retention_mask,
    chunk_scores_to_token_scores,
    hf_cache_to_tuple,
    quantize_kv_layer,
)
from .integrations import quantize_hf_cache
from .profiles import GraphKVProfile, get_profile, list_profiles

__version__ = "0.1.0"

__all__ = [
    "GraphKVProfile",
    "KvQuantConfig",
    "QuantizedKvCache",
    "QuantizedKvLayer",
    "QuantizedTensor",
    "attention_from_kv",
    "attention_report",
    "build_retention_mask",
    "chunk_scores_to_token_scores",
    "get_profile",
    "hf_cache_to_tuple",
    "list_profiles",
    "quantize_hf_cache",
    "quantize_kv_layer",
]
