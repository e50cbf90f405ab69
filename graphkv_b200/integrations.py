"""``quantize_hf_cache`` -- the drop-in entry point (reference:
``src/graphkv/integrations.py:12-62``), same signature, same profile handling,
same output formats."""
from __future__ import annotations

import shlex
from typing import Iterable

from .core import QuantizedKvCache, export_dequantized, hf_cache_to_tuple, roundtrip_host_cache
from .profiles import GraphKVProfile, get_profile


def quantize_hf_cache(
    past_key_values: object,
    profile: str | GraphKVProfile = "graphkv",
    *,
    importance_scores=None,
    graph_memory=None,
    graph_mneme=None,
    graph_mneme_model=None,
    graph_mneme_device: str = "auto",
    output: str = "dynamic",
    model_config: object | None = None,
    max_cache_len: int | None = None,
) -> object:
    """Quantize a Hugging Face cache and export it in the requested format.

    ``output`` is ``compressed`` (the ``QuantizedKvCache``), ``legacy``,
    ``dynamic``, ``static`` or ``sliding_window``.  Explicit
    ``importance_scores`` take precedence over ``graph_memory``; a graph memory
    request is scored with the Graph Mneme model into per-token scores first.
    """
    selected = get_profile(profile)
    if selected.config is None:
        raise ValueError(f"Profile {selected.name!r} is an engine-native recipe, not a GraphKV profile.")
    graph_request = graph_memory if graph_memory is not None else graph_mneme
    if importance_scores is None and graph_request is not None:
        from .graph_model import graph_mneme_request_token_scores

        importance_scores = graph_mneme_request_token_scores(
            _hf_cache_seq_len(past_key_values), graph_request, model=graph_mneme_model, device=graph_mneme_device)
    if output in {"legacy", "dynamic", "static", "sliding_window"}:
        # a cache in pinned host memory: copies in both directions overlap the kernels
        pairs = hf_cache_to_tuple(past_key_values, cache_role="self")
        dequantized = roundtrip_host_cache(pairs, selected.config, importance_scores)
        if dequantized is not None:
            return export_dequantized(dequantized, output, config=model_config, max_cache_len=max_cache_len)
        compressed = QuantizedKvCache.from_past_key_values(pairs, selected.config, importance_scores)
    else:
        compressed = QuantizedKvCache.from_hf_cache(past_key_values, selected.config,
                                                    importance_scores=importance_scores)
    if output == "compressed":
        return compressed
    return compressed.to_hf_cache(output, config=model_config, max_cache_len=max_cache_len)


def _hf_cache_seq_len(past_key_values: object) -> int:
    layers = hf_cache_to_tuple(past_key_values)
    if not layers:
        raise ValueError("past_key_values must contain at least one non-empty KV layer.")
    return int(layers[0][0].shape[2])


# ---------------------------------------------------------------------------
# engine-native recipes (integrations.py:65-124): the settings a vLLM or
# llama.cpp profile stands for, as keyword arguments, CLI flags or environment
# ---------------------------------------------------------------------------

def _engine_profile(profile, engine: str, label: str) -> GraphKVProfile:
    selected = get_profile(profile)
    if selected.engine != engine:
        raise ValueError(f"Profile {selected.name!r} is not a {label} profile.")
    return selected


def vllm_kwargs(profile: str | GraphKVProfile = "vllm-fp8-calibrated", **overrides) -> dict[str, object]:
    """Keyword arguments for ``vllm.LLM(...)``: vLLM's native KV cache dtype and
    scale calibration (low-bit GraphKV caches would need a vLLM backend patch)."""
    selected = _engine_profile(profile, "vllm", "vLLM")
    return {"kv_cache_dtype": selected.vllm_kv_cache_dtype,
            "calculate_kv_scales": selected.vllm_calculate_kv_scales, **overrides}


def vllm_cli_args(profile: str | GraphKVProfile = "vllm-fp8-calibrated") -> list[str]:
    kw = vllm_kwargs(get_profile(profile))
    return ["--kv-cache-dtype", str(kw["kv_cache_dtype"])] + (["--calculate-kv-scales"]
                                                              if kw.get("calculate_kv_scales") else [])


def llama_cpp_args(profile: str | GraphKVProfile = "llamacpp-q8") -> list[str]:
    selected = _engine_profile(profile, "llama.cpp", "llama.cpp")
    return ["--cache-type-k", str(selected.llama_cache_type_k), "--cache-type-v", str(selected.llama_cache_type_v)]


def llama_cpp_env(profile: str | GraphKVProfile = "llamacpp-q8") -> dict[str, str]:
    selected = _engine_profile(profile, "llama.cpp", "llama.cpp")
    return {"LLAMA_ARG_CACHE_TYPE_K": str(selected.llama_cache_type_k),
            "LLAMA_ARG_CACHE_TYPE_V": str(selected.llama_cache_type_v)}


def llama_cpp_command(model_path: str, *, profile: str | GraphKVProfile = "llamacpp-q8", binary: str = "llama-cli",
                      extra_args: Iterable[str] = ()) -> str:
    """Shell-quoted llama.cpp command line with the profile's cache types."""
    return shlex.join([binary, "-m", model_path, *llama_cpp_args(profile), *extra_args])
