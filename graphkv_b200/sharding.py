"""Weak sharding of a KV cache over the GPUs of one node.

The cache shards by (layer, kv-head) unit: keys are grouped over tokens within
(batch, head, channel) and values over channels within (batch, head, token), so
no quantization group crosses a head, and the tier selection depends only on
the [T] importance scores, which every rank recomputes.  The only exchange is
one all-gather of per-shard byte counts, from which every rank derives the
whole cache's statistics.
"""
from __future__ import annotations

import torch


def shard_units(layers: int, heads: int, world: int, rank: int) -> list[tuple[int, int, int]]:
    """Contiguous range of the layers * heads units owned by `rank`, as
    [(layer, first_head, end_head), ...]."""
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    units = layers * heads
    lo, hi = units * rank // world, units * (rank + 1) // world
    out = []
    u = lo
    while u < hi:
        layer, h0 = divmod(u, heads)
        h1 = min(heads, h0 + (hi - u))
        out.append((layer, h0, h1))
        u += h1 - h0
    return out


def shard_bytes(shape: tuple, dtype: torch.dtype, config, has_scores: bool, first_head: int) -> tuple[int, int]:
    """(compressed, original) bytes of one layer shard [B, heads, T, D].  The
    layer's index lists (4 bytes per token) are counted once per layer, by the
    shard that holds head 0, so the shards' sums equal the whole cache's."""
    from .config import layer_memory_bytes, resolve_tiers, tensor_plans

    B, H, T, D = shape
    tiers = resolve_tiers(config, T, has_scores)
    comp = layer_memory_bytes(tuple(shape), dtype, tiers, tensor_plans(config, tuple(shape), tiers))
    if first_head != 0:
        comp -= 4 * T
    esize = torch.empty((), dtype=dtype).element_size()
    return comp, 2 * B * H * T * D * esize


def shard_stats(compressed_bytes: int, original_bytes: int, device=None) -> torch.Tensor:
    """The per-shard vector that is all-gathered: [compressed bytes, original bytes]."""
    return torch.tensor([float(compressed_bytes), float(original_bytes)], dtype=torch.float64, device=device)


def combine_stats(gathered: torch.Tensor) -> dict:
    """Whole-cache statistics from the all-gathered [world * 2] vector."""
    v = gathered.reshape(-1, 2).double()
    compressed, original = float(v[:, 0].sum()), float(v[:, 1].sum())
    return {"memory_bytes": compressed, "original_memory_bytes": original,
            "compression_ratio": original / compressed if compressed else float("inf"),
            "shards": int(v.shape[0])}
