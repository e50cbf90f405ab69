"""A KV cache sharded over the GPUs of one node by (layer, kv-head) unit.

Keys are grouped over tokens within (batch, head, channel) and values over
channels within (batch, head, token), so no quantization group crosses a head,
and the tier selection depends only on the [T] importance scores, which every
rank computes for itself.  Each rank compresses and dequantizes its own units
in its own HBM with no exchange on the data path.  The only collective is one
all-gather of per-layer byte and token counts, from which every rank rebuilds
the whole cache's ``stats()`` -- the same 12 numbers as the unsharded
``QuantizedKvCache.stats()`` (reference core.py:392-413).

A layer split over several ranks is accounted for as the reference accounts for
the whole layer:

* its index lists (4 bytes per token) and its token counts belong to the layer,
  so only the piece holding head 0 reports them;
* the passthrough decision (core.py:770-772) is taken on the whole layer's
  shape, not on a piece's, and applied to every piece of the layer.
"""
from __future__ import annotations

from dataclasses import replace
from typing import Sequence

import torch

from .config import KvQuantConfig, layer_memory_bytes, resolve_tiers, tensor_plans
from .core import QuantizedKvCache, QuantizedKvLayer, _check_pair, _full_precision_layer, _quantize_layers

# per-layer counters of one piece: compressed bytes, original bytes, retained,
# compressed and low-priority tokens
STAT_FIELDS = ("compressed_bytes", "original_bytes", "retained_tokens", "compressed_tokens", "low_priority_tokens")


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


def _esize(dtype: torch.dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


def layer_is_passthrough(shape: tuple, dtype: torch.dtype, config: KvQuantConfig, has_scores: bool) -> bool:
    """The reference's passthrough rule for a whole layer of ``shape`` [B, H, T, D]."""
    B, H, T, D = shape
    tiers = resolve_tiers(config, T, has_scores)
    plans = tensor_plans(config, tuple(shape), tiers)
    return config.skip_if_not_smaller and \
        layer_memory_bytes(tuple(shape), dtype, tiers, plans) >= 2 * B * H * T * D * _esize(dtype)


def shard_bytes(shape: tuple, dtype: torch.dtype, config: KvQuantConfig, has_scores: bool,
                first_head: int) -> tuple[int, int]:
    """(compressed, original) bytes of one compressed piece [B, heads, T, D] of a
    layer, computed on the host; the index lists count only in the head-0 piece."""
    B, H, T, D = shape
    tiers = resolve_tiers(config, T, has_scores)
    comp = layer_memory_bytes(tuple(shape), dtype, tiers, tensor_plans(config, tuple(shape), tiers))
    if first_head != 0:
        comp -= 4 * T
    return comp, 2 * B * H * T * D * _esize(dtype)


def planned_piece_row(piece_shape: tuple, dtype: torch.dtype, config: KvQuantConfig, has_scores: bool,
                      first_head: int, heads: int) -> list[int]:
    """STAT_FIELDS of a piece [B, h, T, D] computed on the host before any kernel
    runs (tier sizes and byte counts do not depend on the data)."""
    B, h, T, D = piece_shape
    head0 = first_head == 0
    original = 2 * B * h * T * D * _esize(dtype)
    if layer_is_passthrough((B, heads, T, D), dtype, config, has_scores):
        return [original, original, T if head0 else 0, 0, 0]
    tiers = resolve_tiers(config, T, has_scores)
    comp = layer_memory_bytes(tuple(piece_shape), dtype, tiers, tensor_plans(config, tuple(piece_shape), tiers))
    if not head0:
        comp -= 4 * T
    return [comp, original, tiers.n_retained if head0 else 0,
            (tiers.n_standard + tiers.n_cold) if head0 else 0, tiers.n_cold if head0 else 0]


def gather_stat_rows(rows: torch.Tensor, group=None, device: torch.device | str | None = None) -> torch.Tensor:
    """Sum of every rank's [layers, 5] counters: one all-gather when a process
    group of more than one rank is initialised (on ``device``: a CUDA device for
    NCCL), the local counters otherwise."""
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        world = dist.get_world_size(group)
        local = rows.to(device) if device is not None else rows
        local = local.contiguous()
        gathered = torch.empty((world * rows.shape[0], rows.shape[1]), dtype=torch.int64, device=local.device)
        dist.all_gather_into_tensor(gathered, local, group=group)
        return gathered.view(world, *rows.shape).sum(dim=0).cpu()
    return rows


def piece_stat_row(layer: QuantizedKvLayer, first_head: int) -> list[int]:
    """STAT_FIELDS of one compressed (or passthrough) piece of a layer."""
    head0 = first_head == 0
    if layer.passthrough_keys is not None:
        T = layer.original_shape[layer.seq_dim]
        nbytes = layer.memory_bytes()
        return [nbytes, layer.original_memory_bytes(), T if head0 else 0, 0, 0]
    comp = layer.memory_bytes()
    if not head0:
        comp -= 4 * layer.original_shape[layer.seq_dim]
    return [comp, layer.original_memory_bytes(),
            layer.retained_token_count() if head0 else 0,
            layer.compressed_token_count() if head0 else 0,
            layer.low_priority_token_count() if head0 else 0]


def stats_from_rows(rows: torch.Tensor) -> dict[str, float]:
    """The reference's cache ``stats()`` (core.py:392-413) from per-layer
    STAT_FIELDS summed over all pieces ([layers, 5] int64)."""
    per_layer = [[int(x) for x in r] for r in rows.tolist()]
    original = sum(r[1] for r in per_layer)
    compressed = sum(r[0] for r in per_layer)
    retained = sum(r[2] for r in per_layer)
    comp_tokens = sum(r[3] for r in per_layer)
    low = sum(r[4] for r in per_layer)
    total = retained + comp_tokens
    ratios = [r[1] / max(r[0], 1) for r in per_layer]
    return {
        "layers": float(len(per_layer)),
        "original_bytes": float(original),
        "compressed_bytes": float(compressed),
        "compression_ratio": original / max(compressed, 1),
        "retained_tokens": float(retained),
        "compressed_tokens": float(comp_tokens),
        "standard_compressed_tokens": float(comp_tokens - low),
        "low_priority_tokens": float(low),
        "retained_fraction": retained / max(total, 1),
        "compressed_fraction": comp_tokens / max(total, 1),
        "min_layer_compression_ratio": min(ratios, default=0.0),
        "max_layer_compression_ratio": max(ratios, default=0.0),
    }


class ShardedKvCache:
    """This rank's pieces of a cache sharded by (layer, kv-head) unit.

    ``units`` lists the pieces as (layer, first_head, end_head); ``local`` holds
    one compressed layer per piece, in the same order.  ``stats()`` gathers the
    per-layer counts of every rank once and returns the whole cache's statistics.
    """

    def __init__(self, local: QuantizedKvCache, units: Sequence[tuple[int, int, int]], n_layers: int):
        if len(local.layers) != len(units):
            raise ValueError("one compressed piece per unit range is required.")
        self.local, self.units, self.n_layers = local, list(units), n_layers

    @classmethod
    def from_past_key_values(cls, pieces: Sequence[tuple[torch.Tensor, torch.Tensor]],
                             units: Sequence[tuple[int, int, int]], n_layers: int, heads: int,
                             config: KvQuantConfig,
                             importance_scores: Sequence[torch.Tensor] | torch.Tensor | None = None
                             ) -> "ShardedKvCache":
        """Compress this rank's pieces: ``pieces[i]`` is (K, V) [B, h1 - h0, T, D]
        of unit range ``units[i]`` of a cache with ``heads`` kv-heads per layer.
        Per-layer scores are indexed by the piece's layer."""
        config.validate()
        units = list(units)
        if len(pieces) != len(units):
            raise ValueError("one (keys, values) piece per unit range is required.")
        keep_all = replace(config, skip_if_not_smaller=False)
        out: list[QuantizedKvLayer | None] = [None] * len(units)
        todo, todo_scores, slots = [], [], []
        for i, ((k, v), (layer, h0, h1)) in enumerate(zip(pieces, units)):
            _check_pair(k, v)
            if k.shape[1] != h1 - h0 or not 0 <= h0 < h1 <= heads or not 0 <= layer < n_layers:
                raise ValueError("piece shape does not match its unit range.")
            s = importance_scores if (importance_scores is None or isinstance(importance_scores, torch.Tensor)) \
                else importance_scores[layer]
            B, _, T, D = k.shape
            if layer_is_passthrough((B, heads, T, D), k.dtype, config, s is not None):
                out[i] = _full_precision_layer(k.detach(), v.detach())
            else:
                todo.append((k, v))
                todo_scores.append(s)
                slots.append(i)
        if todo:
            for i, lay in zip(slots, _quantize_layers(todo, keep_all, todo_scores)):
                out[i] = lay
        return cls(QuantizedKvCache(out), units, n_layers)

    def stat_rows(self) -> torch.Tensor:
        """This rank's per-layer counters, [n_layers, 5] int64 (zero for layers it
        does not hold)."""
        rows = torch.zeros(self.n_layers, len(STAT_FIELDS), dtype=torch.int64)
        for lay, (layer, h0, _) in zip(self.local.layers, self.units):
            rows[layer] += torch.tensor(piece_stat_row(lay, h0), dtype=torch.int64)
        return rows

    def stats(self, group=None, device: torch.device | str | None = None) -> dict[str, float]:
        """Whole-cache statistics: one all-gather of every rank's counters when a
        process group is initialised (on ``device``: a CUDA device for NCCL), the
        local counters alone otherwise."""
        return stats_from_rows(gather_stat_rows(self.stat_rows(), group, device))

    def dequantize(self) -> tuple[tuple[torch.Tensor, torch.Tensor], ...]:
        """Dequantized (K, V) of this rank's pieces, in ``units`` order."""
        return self.local.dequantize()
