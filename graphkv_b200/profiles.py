"""Named profiles (the reference's ``src/graphkv/profiles.py:12-164``: same names,
same policy values, same lookup behaviour)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

from .config import KvQuantConfig

Engine = Literal["graphkv", "vllm", "llama.cpp"]

GRAPHKV_DEFAULT_CONFIG = KvQuantConfig(
    bits=4, group_size=64, residual_length=256, sink_length=128, quantizer="affine",
    long_context_threshold=8192, long_context_quantizer="symmetric",
    key_group_axis="token", value_group_axis="channel",
    semantic_protection_ratio=0.01, semantic_protection_min_context=8192,
    semantic_residual_length=128, semantic_residual_min_context=8192,
    low_priority_ratio=0.25, long_low_priority_ratio=0.35, long_low_priority_min_context=32768,
    low_priority_min_context=8192, low_priority_value_bits=2,
    low_priority_value_rotation="hadamard", low_priority_value_rotation_min_context=32768,
)

QWEN7_NF4_COMPARISON_CONFIG = KvQuantConfig(
    bits=4, group_size=32, residual_length=512, sink_length=128, quantizer="affine",
    long_context_threshold=8192, long_context_quantizer="symmetric",
    key_group_axis="token", value_group_axis="channel",
    semantic_protection_ratio=0.02, semantic_protection_min_context=8192,
)


@dataclass(frozen=True)
class GraphKVProfile:
    name: str
    engine: Engine
    description: str
    config: KvQuantConfig | None = None
    vllm_kv_cache_dtype: str | None = None
    vllm_calculate_kv_scales: bool | None = None
    llama_cache_type_k: str | None = None
    llama_cache_type_v: str | None = None

    @property
    def is_native_graphkv(self) -> bool:
        return self.engine == "graphkv"


PROFILES: dict[str, GraphKVProfile] = {
    "graphkv": GraphKVProfile("graphkv", "graphkv",
                              "Default GraphKV profile with built-in Mneme-guided retention and tiering.",
                              GRAPHKV_DEFAULT_CONFIG),
    "graphkv-int2-max": GraphKVProfile(
        "graphkv-int2-max", "graphkv", "Maximum compression profile for Transformers cache experiments.",
        KvQuantConfig(bits=2, group_size=128, residual_length=0, quantizer="affine",
                      key_group_axis="token", value_group_axis="channel")),
    "graphkv-int4-balanced": GraphKVProfile(
        "graphkv-int4-balanced", "graphkv", "Balanced profile for grouped-query models such as Qwen2.",
        KvQuantConfig(bits=4, group_size=64, residual_length=0, quantizer="symmetric",
                      key_group_axis="token", value_group_axis="channel")),
    "graphkv-int4-safe": GraphKVProfile(
        "graphkv-int4-safe", "graphkv", "Safer 4-bit profile with a recent residual tail and outlier retention.",
        KvQuantConfig(bits=4, group_size=64, residual_length=96, sink_length=32, quantizer="symmetric",
                      key_group_axis="token", value_group_axis="channel",
                      outlier_protection_ratio=0.02, min_outlier_tokens=1)),
    "graphkv-qwen7-nf4": GraphKVProfile(
        "graphkv-qwen7-nf4", "graphkv", "Conservative Qwen2.5-7B NF4 profile used for local comparison rows.",
        QWEN7_NF4_COMPARISON_CONFIG),
    "vllm-fp8": GraphKVProfile("vllm-fp8", "vllm", "Native vLLM FP8 KV cache with default scales.",
                               vllm_kv_cache_dtype="fp8", vllm_calculate_kv_scales=False),
    "vllm-fp8-calibrated": GraphKVProfile("vllm-fp8-calibrated", "vllm",
                                          "Native vLLM FP8 KV cache with warmup scale calculation.",
                                          vllm_kv_cache_dtype="fp8", vllm_calculate_kv_scales=True),
    "llamacpp-q8": GraphKVProfile("llamacpp-q8", "llama.cpp", "Native llama.cpp Q8_0 KV cache. Usually conservative.",
                                  llama_cache_type_k="q8_0", llama_cache_type_v="q8_0"),
    "llamacpp-q4": GraphKVProfile("llamacpp-q4", "llama.cpp", "Native llama.cpp Q4_0 KV cache. More aggressive.",
                                  llama_cache_type_k="q4_0", llama_cache_type_v="q4_0"),
}


def get_profile(name: str | GraphKVProfile) -> GraphKVProfile:
    """profiles.py:153-160: objects pass through, unknown names raise KeyError."""
    if isinstance(name, GraphKVProfile):
        return name
    try:
        return PROFILES[name]
    except KeyError as exc:
        choices = ", ".join(sorted(PROFILES))
        raise KeyError(f"Unknown GraphKV profile {name!r}. Choices: {choices}") from exc


def list_profiles() -> tuple[GraphKVProfile, ...]:
    return tuple(PROFILES.values())
