"""Seeded synthetic KV caches with the shapes and value distributions of the
workloads this library is measured and checked on.

No public dataset is involved: the caches are random tensors with
Qwen2.5 / GPT-2 shaped geometry.

* keys: N(0, 1) scaled per (layer, head, channel) by exp(N(0, 1)) -- a
  log-normal channel scale, as real key caches have (GPT-2 shaped cache: plain
  N(0, 1) with 4 random channels per head scaled by 15 as outliers);
* values: N(0, 1);
* importance scores: exp(2 * N(0, 1)) as fp32 ``[T]`` from seed 99, shared by
  every layer and batch row.

CPU generation (``device="cpu"``) is bit-reproducible on any x86 host with the
same torch build; it is what the parity tests use.  ``device="cuda"`` draws
from a CUDA generator (different values, same distributions) and is what the
throughput benchmark uses for its multi-GB inputs.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

SCORES_SEED = 99


@dataclass(frozen=True)
class Workload:
    key: str
    name: str
    layers: int
    heads: int
    head_dim: int
    batch: int
    seq: int
    dtype: torch.dtype
    profile: str
    with_scores: bool
    outlier_channels: int = 0      # > 0 selects the GPT-2 style key outliers
    outlier_scale: float = 15.0
    seed: int = 1234

    @property
    def shape(self) -> tuple[int, int, int, int]:
        return (self.batch, self.heads, self.seq, self.head_dim)

    @property
    def input_bytes(self) -> int:
        b, h, t, d = self.shape
        return 2 * self.layers * b * h * t * d * torch.empty((), dtype=self.dtype).element_size()


WORKLOADS = {
    "gpt2-1k": Workload("gpt2-1k", "GPT-2-small shaped, 1k tokens, fp32", 12, 12, 64, 1, 1024,
                        torch.float32, "graphkv-int2-max", False, outlier_channels=4),
    "qwen0.5b-4k": Workload("qwen0.5b-4k", "Qwen2.5-0.5B shaped, 4k tokens, bf16", 24, 2, 64, 1, 4096,
                            torch.bfloat16, "graphkv-int4-balanced", False),
    "qwen7b-16k": Workload("qwen7b-16k", "Qwen2.5-7B shaped, 16k tokens, bf16", 28, 4, 128, 1, 16384,
                           torch.bfloat16, "graphkv", True),
    "qwen7b-32k": Workload("qwen7b-32k", "Qwen2.5-7B shaped, 32k tokens, bf16", 28, 4, 128, 1, 32768,
                           torch.bfloat16, "graphkv", True),
    "qwen7b-8x131k": Workload("qwen7b-8x131k", "Qwen2.5-7B shaped, batch 8 x 131k tokens, bf16", 28, 4, 128, 8,
                              131072, torch.bfloat16, "graphkv", True),
}


def _generator(device: str, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_layer(w: Workload, layer: int, device: str = "cpu", batch=None, heads=None):
    """Keys and values ``[B, H, T, D]`` of one layer.  ``batch``/``heads`` select
    a sub-range (``range`` objects) of the full layer, generated so that a
    sub-range is identical to the same slice of the full layer."""
    B, H, T, D = w.shape
    batch = range(B) if batch is None else batch
    heads = range(H) if heads is None else heads
    g = _generator(device, w.seed * 1000 + layer)
    # one scale draw per layer so that slices agree with the full tensor
    if w.outlier_channels:
        scale = torch.ones(H, D, device=device)
        for h in range(H):
            ch = torch.randperm(D, generator=g, device=device)[: w.outlier_channels]
            scale[h, ch] = w.outlier_scale
    else:
        scale = torch.exp(torch.randn(H, D, generator=g, device=device))
    ks, vs = [], []
    for b in batch:
        kh, vh = [], []
        for h in heads:
            gk = _generator(device, (w.seed * 1000 + layer) * 4096 + b * 64 + h)
            k = torch.randn(T, D, generator=gk, device=device) * scale[h]
            v = torch.randn(T, D, generator=gk, device=device)
            kh.append(k.to(w.dtype))
            vh.append(v.to(w.dtype))
        ks.append(torch.stack(kh))
        vs.append(torch.stack(vh))
    return torch.stack(ks).contiguous(), torch.stack(vs).contiguous()


def make_scores(w: Workload, device: str = "cpu"):
    if not w.with_scores:
        return None
    g = _generator(device, SCORES_SEED)
    return torch.exp(2.0 * torch.randn(w.seq, generator=g, device=device))


def make_cache(w: Workload, device: str = "cpu"):
    """Legacy tuple cache ``((K, V), ...)`` of all layers."""
    return tuple(make_layer(w, l, device) for l in range(w.layers))
