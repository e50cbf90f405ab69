"""``quantize_hf_cache`` -- the drop-in entry point (reference:
``src/graphkv/integrations.py:12-62``), same signature, same profile handling,
same output formats."""
from __future__ import annotations

from .core import QuantizedKvCache, hf_cache_to_tuple
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
    compressed = QuantizedKvCache.from_hf_cache(past_key_values, selected.config, importance_scores=importance_scores)
    if output == "compressed":
        return compressed
    return compressed.to_hf_cache(output, config=model_config, max_cache_len=max_cache_len)


def _hf_cache_seq_len(past_key_values: object) -> int:
    layers = hf_cache_to_tuple(past_key_values)
    if not layers:
        raise ValueError("past_key_values must contain at least one non-empty KV layer.")
    return int(layers[0][0].shape[2])
