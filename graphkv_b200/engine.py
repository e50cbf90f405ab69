"""Prepared compression of a fixed cache geometry: plan once, run many.

``CompressionEngine(pairs, config, scores)`` resolves the policy, allocates the
device arena of every stored tensor and the dequantized outputs, and builds the
C plans once.  Each ``quantize()`` then issues, per run of same-shaped layers,
one selection launch and, per 40 layers, one quantize launch per kernel variant
(grouping axis x rotation) that each tensor's tiers use -- keys: one; values:
two when the cold tier is rotated; ``dequantize()`` issues the same number of
dequantize launches -- no allocation, no Python object construction.  The
inputs are read at their current addresses on every call, so callers refill
them in place (e.g. a serving loop that compresses caches of one shape).

``cache()`` returns a ``QuantizedKvCache`` whose tensors are views into the
engine's arena (valid until the next ``quantize()``).
"""
from __future__ import annotations

import torch

from .config import KvQuantConfig
from .core import QuantizedKvCache, _check_pair, _prepare_group


class CompressionEngine:
    def __init__(self, pairs, config: KvQuantConfig, importance_scores=None):
        config.validate()
        pairs = list(pairs)
        for k, v in pairs:
            _check_pair(k, v)
        per_layer = [importance_scores if (importance_scores is None or isinstance(importance_scores, torch.Tensor))
                     else importance_scores[i] for i in range(len(pairs))]
        self.items = []
        i = 0
        while i < len(pairs):
            j = i + 1
            while (j < len(pairs) and pairs[j][0].shape == pairs[i][0].shape and pairs[j][0].dtype == pairs[i][0].dtype
                   and per_layer[j] is per_layer[i]):
                j += 1
            self.items.extend(_prepare_group(pairs[i:j], config, per_layer[i]))
            i = j

    @property
    def runs(self):
        return [it[1] for it in self.items if it[0] == "run"]

    def launches_per_step(self) -> int:
        """Kernel launches of one quantize() + dequantize() (for the fast path of every run):
        per tensor, one tile launch per distinct (axis, rotation) among its non-empty tiers."""
        n = 0
        for it in self.items:
            if it[0] != "run":
                continue
            run = it[1]
            plan = run.plan
            variants = 0
            for tensor in range(2):
                kinds = set()
                for tier, count in ((0, plan.n_standard), (2, plan.n_cold)):
                    if count > 0:
                        spec = plan.spec[tier + tensor]
                        kinds.add((spec.axis, bool(spec.rotation)))
                variants += max(1, len(kinds))
            chunks = -(-len(run.pairs) // 40)  # gkv_quantize splits calls into 40-layer launches
            n += (1 if it[3] else 0) + (1 if run.outlier is not None else 0) + variants * chunks + variants
        return n

    def quantize(self) -> None:
        for it in self.items:
            if it[0] == "run":
                _, run, s, needs_select = it
                if needs_select:
                    run.select(s)
                run.quantize()

    def dequantize(self) -> None:
        for run in self.runs:
            run.dequantize()

    def cache(self) -> QuantizedKvCache:
        layers = []
        for it in self.items:
            layers.extend([it[1]] if it[0] == "pass" else it[1].layers())
        return QuantizedKvCache(layers)

    def outputs(self) -> list:
        out = []
        for it in self.items:
            if it[0] == "pass":
                out.append((it[1].passthrough_keys, it[1].passthrough_values))
            else:
                run = it[1]
                out.extend((run.out_k[l], run.out_v[l]) for l in range(len(run.pairs)))
        return out
