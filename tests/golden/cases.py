"""Golden cases: seeded inputs whose reference outputs are recorded in
``tests/golden/*.json`` / ``*.npz`` by ``make_golden.py``.

Each case names a profile (optionally with field overrides), a cache geometry,
an input recipe and a scores recipe.  The same builder regenerates the inputs
bit-for-bit wherever the tests run, so only the reference's OUTPUTS are stored:
full arrays for small cases, SHA-256 digests for the full-size workloads.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np
import torch

from graphkv_b200.workloads import WORKLOADS, make_layer, make_scores

DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@dataclass(frozen=True)
class Case:
    name: str
    profile: str
    shape: tuple = (1, 2, 256, 64)          # B, H, T, D
    dtype: str = "bf16"
    layers: int = 1
    keys: str = "lognormal"                 # lognormal | outlier | constant | zeros | smallrange
    scores: str = "none"                    # none | lognormal | ties | batch | heads | per_layer
    overrides: dict = field(default_factory=dict)
    seed: int = 7
    workload: str = ""                      # full-size workload key (digest-only case)
    layer_subset: tuple = ()                # layers of the workload to record (empty = all)
    full_arrays: bool = True                # store whole arrays (small cases) or digests only
    score_rows: int = 0                     # rows_adv / tx_adv: size of the averaged dimension


def _gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def case_layers(c: Case):
    """List of (K, V) CPU tensors for the case."""
    if c.workload:
        w = WORKLOADS[c.workload]
        idx = c.layer_subset or tuple(range(w.layers))
        return [make_layer(w, l) for l in idx]
    B, H, T, D = c.shape
    dt = DTYPES[c.dtype]
    out = []
    for l in range(c.layers):
        g = _gen(c.seed * 100 + l)
        if c.keys == "lognormal":
            k = torch.randn(B, H, T, D, generator=g) * torch.exp(torch.randn(H, 1, D, generator=g))
        elif c.keys == "outlier":
            k = torch.randn(B, H, T, D, generator=g)
            for h in range(H):
                ch = torch.randperm(D, generator=g)[: min(4, D)]
                k[:, h, :, ch] *= 15.0
        elif c.keys == "constant":
            # constant rows/columns make affine ranges degenerate (core.py:869-877)
            k = torch.full((B, H, T, D), -0.75)
            k[:, :, ::3, :] = 0.5
            k[:, :, :, ::5] = 0.0
        elif c.keys == "zeros":
            k = torch.zeros(B, H, T, D)
        elif c.keys == "tiny":
            # values rows scaled toward the bottom of the fp32 range, with -0 entries:
            # the rotated paths must divide these exactly
            k = torch.randn(B, H, T, D, generator=g)
        elif c.keys == "smallrange":
            # tiny positive offsets: ranges below 1e-8 and min > 0
            k = 3.0 + torch.randn(B, H, T, D, generator=g) * 1e-9
        else:
            raise ValueError(c.keys)
        v = torch.randn(B, H, T, D, generator=g)
        if c.keys == "zeros":
            v[:, :, 1::2, :] = 0.0
        if c.keys == "tiny":
            v[:, :, ::3, :] *= 2.0 ** -100
            v[:, :, 1::7, 5] = -0.0
            v[:, :, 2::5, :] = -0.0
        out.append((k.to(dt).contiguous(), v.to(dt).contiguous()))
    return out


def case_scores(c: Case):
    """Importance scores (tensor, per-layer list, or None)."""
    if c.workload:
        return make_scores(WORKLOADS[c.workload])
    B, H, T, D = c.shape
    g = _gen(c.seed + 99)
    if c.scores == "none":
        return None
    if c.scores == "lognormal":
        return torch.exp(2.0 * torch.randn(T, generator=g))
    if c.scores == "ties":
        # few distinct values: ties straddle every selection boundary
        return torch.randint(0, 4, (T,), generator=g).to(torch.float32)
    if c.scores == "batch":
        return torch.exp(torch.randn(B, T, generator=g))
    if c.scores == "heads":
        return torch.exp(torch.randn(H, T, generator=g))
    if c.scores == "per_layer":
        return [torch.exp(2.0 * torch.randn(T, generator=g)) for _ in range(c.layers)]
    if c.scores in ("rows_adv", "tx_adv", "rows3_adv"):
        vals = adversarial_score_rows(T, c.score_rows, g)  # [T, R]
        if c.scores == "tx_adv":
            return vals.contiguous()
        rows = vals.t().contiguous()
        return rows.reshape(2, c.score_rows // 2, T) if c.scores == "rows3_adv" else rows
    raise ValueError(c.scores)


def adversarial_score_rows(T: int, R: int, g: torch.Generator) -> torch.Tensor:
    """[T, R] fp32 scores whose per-token means tie in exact arithmetic within a
    few levels and differ only through fp32 rounding: every token's R values are
    one fixed multiset of magnitudes from 1e-2 to 1e4 with alternating signs, in
    a different order per token, plus one of six base levels.  The selection
    boundaries fall inside a level, so which tokens are kept is decided by the
    order of the fp32 additions of the mean."""
    mags = torch.pow(10.0, torch.rand(R, generator=g, dtype=torch.float64) * 6.0 - 2.0)
    signs = torch.where(torch.arange(R) % 2 == 0, 1.0, -1.0).double()
    multiset = (mags * signs).float()
    base = 1.0 + 0.25 * torch.randint(0, 6, (T,), generator=g).float()
    order = torch.argsort(torch.rand(T, R, generator=g), dim=1)
    return multiset[order] + base[:, None]


def tensor_digest(arr: np.ndarray) -> str:
    a = np.ascontiguousarray(arr)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(tuple(a.shape)).encode())
    h.update(a.tobytes())
    return h.hexdigest()


def bits_of(t: torch.Tensor) -> np.ndarray:
    """Storage bit patterns of a tensor as a numpy array (bf16/f16 -> uint16, f32 -> uint32)."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy().view(np.uint32)
    return t.numpy()


CASES = [
    # --- small cases, full arrays -------------------------------------------------------
    Case("int2max_fp32", "graphkv-int2-max", (1, 2, 1024, 64), "f32", layers=2, keys="outlier"),
    Case("int4bal_bf16", "graphkv-int4-balanced", (1, 2, 4096, 64), "bf16", layers=1),
    Case("graphkv_8k_scores", "graphkv", (1, 1, 8192, 64), "bf16", scores="lognormal"),
    Case("graphkv_1k_noscores", "graphkv", (1, 2, 1024, 128), "bf16"),
    Case("graphkv_32k_rot", "graphkv", (1, 1, 32768, 128), "bf16", scores="lognormal", full_arrays=False),
    Case("nf4_affine_1k", "graphkv-qwen7-nf4", (1, 2, 1024, 128), "bf16"),
    Case("nf4_9k_scores", "graphkv-qwen7-nf4", (1, 1, 9000, 64), "bf16", scores="lognormal"),
    Case("int4safe_outlier", "graphkv-int4-safe", (2, 2, 600, 64), "bf16", keys="outlier"),
    Case("fp16_input", "graphkv-int4-balanced", (1, 2, 300, 64), "f16"),
    Case("batch2", "graphkv", (2, 2, 700, 64), "bf16"),
    Case("single_token", "graphkv-int4-balanced", (1, 1, 1, 64), "bf16"),
    Case("odd_tier_37", "graphkv-int4-balanced", (1, 2, 37, 64), "bf16"),
    Case("odd_dim_48", "graphkv-int4-balanced", (1, 2, 130, 48), "bf16"),
    Case("pad_dim_96", "graphkv-int4-balanced", (1, 1, 200, 96), "bf16"),
    Case("tiny_dim_3", "graphkv-int2-max", (1, 1, 50, 3), "f32"),
    Case("affine_degenerate", "graphkv-int2-max", (1, 1, 300, 64), "bf16", keys="constant"),
    Case("affine_smallrange", "graphkv-int2-max", (1, 1, 256, 32), "f32", keys="smallrange"),
    Case("zeros", "graphkv-int4-balanced", (1, 1, 128, 64), "bf16", keys="zeros"),
    Case("all_retained", "graphkv", (1, 1, 200, 64), "bf16", overrides={"skip_if_not_smaller": False}),
    Case("passthrough", "graphkv-int4-balanced", (1, 1, 16, 8), "bf16", overrides={"bits": 8, "group_size": 1}),
    Case("bits8", "graphkv-int4-balanced", (1, 2, 256, 64), "bf16", overrides={"bits": 8}),
    Case("unpacked4", "graphkv-int4-balanced", (1, 2, 256, 64), "bf16", overrides={"pack_int4": False}),
    Case("swapped_axes_rot", "graphkv-int4-balanced", (1, 2, 192, 64), "bf16",
         overrides={"key_group_axis": "channel", "value_group_axis": "token", "rotation": "hadamard"}),
    Case("affine_sink_tail", "graphkv-int4-balanced", (1, 2, 2048, 128), "bf16",
         overrides={"quantizer": "affine", "sink_length": 64, "residual_length": 128}),
    # rotated channel-axis values over 128 channels: two threads per row in the tile kernels
    Case("rot128_int4_sym", "graphkv-int4-balanced", (1, 2, 512, 128), "bf16", overrides={"rotation": "hadamard"}),
    Case("rot128_affine_gs128", "graphkv-int4-balanced", (1, 1, 384, 128), "bf16",
         overrides={"rotation": "hadamard", "quantizer": "affine", "group_size": 128}),
    Case("rot128_int8_f16", "graphkv-int4-balanced", (1, 1, 256, 128), "f16",
         overrides={"rotation": "hadamard", "bits": 8}),
    Case("rot128_int2_gs128", "graphkv-int4-balanced", (1, 2, 512, 128), "bf16",
         overrides={"rotation": "hadamard", "bits": 2, "group_size": 128}),
    Case("rot128_int2_zeros", "graphkv-int4-balanced", (1, 1, 256, 128), "bf16", keys="zeros",
         overrides={"rotation": "hadamard", "bits": 2}),
    Case("rot128_int2_tiny", "graphkv-int4-balanced", (1, 1, 320, 128), "bf16", keys="tiny",
         overrides={"rotation": "hadamard", "bits": 2}),
    Case("scale_bf16", "graphkv-int4-balanced", (1, 1, 256, 64), "bf16", overrides={"scale_dtype": "bf16"}),
    Case("scale_f32_affine", "graphkv-int2-max", (1, 1, 256, 64), "bf16", overrides={"scale_dtype": "f32"}),
    Case("scores_batch", "graphkv", (2, 1, 8192, 64), "bf16", scores="batch"),
    Case("scores_heads", "graphkv", (1, 2, 8192, 64), "bf16", scores="heads"),
    Case("scores_per_layer", "graphkv", (1, 1, 8192, 64), "bf16", layers=2, scores="per_layer"),
    Case("scores_ties", "graphkv", (1, 1, 8192, 64), "bf16", scores="ties"),
    Case("scores_rows64_adv", "graphkv", (1, 1, 8192, 64), "bf16", scores="rows_adv", score_rows=64),
    Case("scores_rows8_tail5", "graphkv", (1, 1, 8197, 64), "bf16", scores="rows_adv", score_rows=8),
    Case("scores_rows3d_adv", "graphkv", (1, 2, 8192, 64), "bf16", scores="rows3_adv", score_rows=48),
    Case("scores_tx27_adv", "graphkv", (1, 1, 8192, 64), "bf16", scores="tx_adv", score_rows=27),
    Case("scores_tx5_adv", "graphkv", (1, 1, 8192, 64), "bf16", scores="tx_adv", score_rows=5),
    Case("cold_bits_mix", "graphkv", (1, 1, 8192, 64), "bf16", scores="lognormal",
         overrides={"low_priority_bits": 2, "low_priority_key_bits": 8, "group_size": 32}),
    # --- full-size workloads, digests only ------------------------------------------------
    Case("w_gpt2_1k", "graphkv-int2-max", workload="gpt2-1k", full_arrays=False),
    Case("w_qwen05b_4k", "graphkv-int4-balanced", workload="qwen0.5b-4k", full_arrays=False),
    Case("w_qwen7b_16k", "graphkv", workload="qwen7b-16k", full_arrays=False),
    Case("w_qwen7b_32k", "graphkv", workload="qwen7b-32k", full_arrays=False),
    Case("w_qwen7b_8x131k_l0", "graphkv", workload="qwen7b-8x131k", layer_subset=(0,), full_arrays=False),
]

CASE_BY_NAME = {c.name: c for c in CASES}
