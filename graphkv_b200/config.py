"""Quantization policy: ``KvQuantConfig`` with the reference's fields, defaults and
validation messages (``src/graphkv/core.py:17-127``), plus the resolution of one
policy into per-layer tier sizes and tensor specs for the CUDA kernels.

Everything here is host arithmetic on Python ints/floats: the tier sizes of a
selection depend only on T and the policy, so they are known before any kernel
runs (the reference learns them from ``nonzero`` after the fact).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Optional

import torch

from . import _lib as L


@dataclass(frozen=True)
class KvQuantConfig:
    """Configuration for group-wise KV-cache quantization.

    Layout of K/V is [batch, heads, tokens, head_dim].  Keys are grouped over
    tokens and values over head_dim channels by default; a prompt sink and a
    recent tail stay in full precision, importance scores can protect more
    tokens and send the least important ones to a low-bit cold tier.
    """

    bits: int = 4
    key_bits: Optional[int] = None
    value_bits: Optional[int] = None
    group_size: int = 64
    residual_length: int = 128
    sink_length: int = 0
    quantizer: str = "symmetric"
    long_context_threshold: Optional[int] = None
    long_context_quantizer: Optional[str] = None
    key_group_axis: str = "token"
    value_group_axis: str = "channel"
    semantic_protection_ratio: float = 0.0
    min_protected_tokens: int = 0
    semantic_protection_min_context: int = 0
    semantic_residual_length: Optional[int] = None
    semantic_residual_min_context: int = 0
    low_priority_ratio: float = 0.0
    long_low_priority_ratio: Optional[float] = None
    long_low_priority_min_context: int = 0
    min_low_priority_tokens: int = 0
    low_priority_min_context: int = 0
    low_priority_bits: Optional[int] = None
    low_priority_key_bits: Optional[int] = None
    low_priority_value_bits: Optional[int] = None
    rotation: str = "none"
    low_priority_value_rotation: Optional[str] = None
    low_priority_value_rotation_min_context: int = 0
    outlier_protection_ratio: float = 0.0
    min_outlier_tokens: int = 0
    pack_int4: bool = True
    scale_dtype: torch.dtype = torch.float16
    skip_if_not_smaller: bool = True

    def validate(self) -> None:
        """Range checks of core.py:60-127 (same messages)."""
        def _bits(name, v, optional):
            if optional and v is None:
                return
            if v not in {2, 4, 8}:
                raise ValueError(f"{name} must be 2, 4, 8, or None." if optional
                                 else f"{name} must be 2, 4, or 8 for this implementation.")

        _bits("bits", self.bits, False)
        _bits("key_bits", self.key_bits, True)
        _bits("value_bits", self.value_bits, True)
        for name in ("group_size",):
            if getattr(self, name) < 1:
                raise ValueError("group_size must be >= 1.")
        for name in ("residual_length", "sink_length"):
            if getattr(self, name) < 0:
                raise ValueError(f"{name} must be >= 0.")
        if self.quantizer not in {"symmetric", "affine"}:
            raise ValueError("quantizer must be 'symmetric' or 'affine'.")
        if self.long_context_threshold is not None and self.long_context_threshold < 1:
            raise ValueError("long_context_threshold must be >= 1 or None.")
        if self.long_context_quantizer is not None and self.long_context_quantizer not in {"symmetric", "affine"}:
            raise ValueError("long_context_quantizer must be 'symmetric', 'affine', or None.")
        if self.key_group_axis not in {"token", "channel"}:
            raise ValueError("key_group_axis must be 'token' or 'channel'.")
        if self.value_group_axis not in {"token", "channel"}:
            raise ValueError("value_group_axis must be 'token' or 'channel'.")
        if not 0.0 <= self.semantic_protection_ratio <= 1.0:
            raise ValueError("semantic_protection_ratio must be in [0, 1].")
        for name in ("min_protected_tokens", "semantic_protection_min_context"):
            if getattr(self, name) < 0:
                raise ValueError(f"{name} must be >= 0.")
        if self.semantic_residual_length is not None and self.semantic_residual_length < 0:
            raise ValueError("semantic_residual_length must be >= 0 or None.")
        if self.semantic_residual_min_context < 0:
            raise ValueError("semantic_residual_min_context must be >= 0.")
        if not 0.0 <= self.low_priority_ratio <= 1.0:
            raise ValueError("low_priority_ratio must be in [0, 1].")
        if self.long_low_priority_ratio is not None and not 0.0 <= self.long_low_priority_ratio <= 1.0:
            raise ValueError("long_low_priority_ratio must be in [0, 1] or None.")
        for name in ("long_low_priority_min_context", "min_low_priority_tokens", "low_priority_min_context"):
            if getattr(self, name) < 0:
                raise ValueError(f"{name} must be >= 0.")
        _bits("low_priority_bits", self.low_priority_bits, True)
        _bits("low_priority_key_bits", self.low_priority_key_bits, True)
        _bits("low_priority_value_bits", self.low_priority_value_bits, True)
        if self.rotation not in {"none", "hadamard"}:
            raise ValueError("rotation must be 'none' or 'hadamard'.")
        if self.low_priority_value_rotation is not None and self.low_priority_value_rotation not in {"none", "hadamard"}:
            raise ValueError("low_priority_value_rotation must be 'none', 'hadamard', or None.")
        if self.low_priority_value_rotation_min_context < 0:
            raise ValueError("low_priority_value_rotation_min_context must be >= 0.")
        if not 0.0 <= self.outlier_protection_ratio <= 1.0:
            raise ValueError("outlier_protection_ratio must be in [0, 1].")
        if self.min_outlier_tokens < 0:
            raise ValueError("min_outlier_tokens must be >= 0.")


# ---------------------------------------------------------------------------
# policy resolution
# ---------------------------------------------------------------------------

def effective_quant_config(config: KvQuantConfig, seq_len: int) -> KvQuantConfig:
    """core.py:913-920: the long-context quantizer switch."""
    if (config.long_context_threshold is not None and config.long_context_quantizer is not None
            and seq_len >= config.long_context_threshold):
        return replace(config, quantizer=config.long_context_quantizer)
    return config


def effective_low_priority_ratio(config: KvQuantConfig, seq_len: int) -> float:
    """core.py:923-929."""
    if config.long_low_priority_ratio is not None and seq_len >= config.long_low_priority_min_context:
        return config.long_low_priority_ratio
    return config.low_priority_ratio


def effective_cold_value_rotation(config: KvQuantConfig, seq_len: int, fallback: str) -> str:
    """core.py:932-942."""
    if config.low_priority_value_rotation is not None and seq_len >= config.low_priority_value_rotation_min_context:
        return config.low_priority_value_rotation
    return fallback


def keep_count(n: int, ratio: float, minimum: int) -> int:
    """min(n, max(ceil(n * ratio), minimum)) -- core.py:1044 and 702-705."""
    return min(n, max(math.ceil(n * ratio), minimum))


@dataclass(frozen=True)
class TierSizes:
    """Selection of one layer, resolved on the host."""
    seq_len: int
    sink: int
    tail: int
    keep_protect: int
    keep_outlier: int
    keep_cold: int
    n_retained: int
    n_standard: int
    n_cold: int

    def policy(self) -> L.SelectPolicy:
        return L.SelectPolicy(self.seq_len, self.sink, self.tail, self.keep_protect, self.keep_outlier,
                              self.keep_cold, self.n_retained, self.n_standard, self.n_cold, 0)


def resolve_tiers(config: KvQuantConfig, seq_len: int, has_scores: bool) -> TierSizes:
    """Tier sizes for T = seq_len: sink/tail (core.py:612-626), importance
    protection (core.py:628-643), outlier protection (core.py:670-679) and the
    cold tier (core.py:685-712)."""
    T = seq_len
    sink = min(config.sink_length, T)
    residual = config.residual_length
    if has_scores and config.semantic_residual_length is not None and T >= config.semantic_residual_min_context:
        residual = config.semantic_residual_length
    tail = min(residual, T)
    union = min(T, sink + tail)
    n_cand = T - union
    keep_protect = 0
    if has_scores and T >= config.semantic_protection_min_context and n_cand > 0:
        keep_protect = max(0, keep_count(n_cand, config.semantic_protection_ratio, config.min_protected_tokens))
    n_cand -= keep_protect
    keep_outlier = 0
    if config.outlier_protection_ratio > 0.0 or config.min_outlier_tokens > 0:
        keep_outlier = max(0, keep_count(n_cand, config.outlier_protection_ratio, config.min_outlier_tokens))
    n_cand -= keep_outlier
    keep_cold = 0
    ratio = effective_low_priority_ratio(config, T)
    if (has_scores and T >= config.low_priority_min_context
            and (ratio > 0.0 or config.min_low_priority_tokens > 0)
            and (config.low_priority_bits is not None or config.low_priority_key_bits is not None
                 or config.low_priority_value_bits is not None)
            and n_cand > 0):
        keep_cold = max(0, keep_count(n_cand, ratio, config.min_low_priority_tokens))
    n_ret = union + keep_protect + keep_outlier
    return TierSizes(T, sink, tail, keep_protect, keep_outlier, keep_cold, n_ret, T - n_ret - keep_cold, keep_cold)


SCALE_DTYPE_CODE = {torch.float16: L.GKV_F16, torch.bfloat16: L.GKV_BF16, torch.float32: L.GKV_F32}


@dataclass(frozen=True)
class TensorPlan:
    """How one compressed tensor is stored (mirrors the QuantizedTensor fields)."""
    bits: int
    quantizer: str
    axis: int            # 2 (token) or 3 (head_dim), as in the reference
    group_size: int      # effective: min(configured, axis length)
    rotation: str
    packed: bool
    scale_dtype: torch.dtype
    n: int               # tier length
    B: int
    H: int
    D: int

    @property
    def axis_len(self) -> int:
        return self.n if self.axis == 2 else self.D

    @property
    def padded(self) -> int:
        return (-self.axis_len) % self.group_size

    @property
    def q_shape(self) -> tuple:
        """Shape of the moved, padded code tensor (core.py:852-859)."""
        if self.axis == 2:
            return (self.B, self.H, self.D, self.n + self.padded)
        return (self.B, self.H, self.n, self.D + self.padded)

    @property
    def numel(self) -> int:
        B, H, a, b = self.q_shape
        return B * H * a * b

    @property
    def sbits(self) -> int:
        return self.bits if self.packed else 8

    @property
    def code_bytes(self) -> int:
        return (self.numel * self.bits + 7) // 8 if self.packed else self.numel

    @property
    def scales_shape(self) -> tuple:
        B, H, a, b = self.q_shape
        return (B, H, a, b // self.group_size, 1)

    @property
    def n_groups(self) -> int:
        return self.numel // self.group_size

    @property
    def slice_bits_aligned(self) -> bool:
        _, _, a, b = self.q_shape
        return (a * b * self.sbits) % 8 == 0

    def memory_bytes(self) -> int:
        """core.py:150-151: codes + scales + zero points."""
        n = self.code_bytes + self.n_groups * torch.empty((), dtype=self.scale_dtype).element_size()
        if self.quantizer == "affine":
            n += self.n_groups
        return n

    def spec(self) -> L.TensorSpec:
        return L.TensorSpec(self.bits, L.GKV_AFFINE if self.quantizer == "affine" else L.GKV_SYMMETRIC,
                            L.GKV_AXIS_TOKEN if self.axis == 2 else L.GKV_AXIS_CHANNEL, self.group_size,
                            L.GKV_ROT_HADAMARD if self.rotation == "hadamard" else L.GKV_ROT_NONE,
                            1 if self.packed else 0, SCALE_DTYPE_CODE[self.scale_dtype], 0)


def tensor_plans(config: KvQuantConfig, shape: tuple, tiers: TierSizes) -> list:
    """The four tensor plans (std K, std V, cold K, cold V; None for an empty
    tier) following core.py:728-755."""
    B, H, T, D = shape
    qc = effective_quant_config(config, T)
    key_axis = 2 if config.key_group_axis == "token" else 3
    value_axis = 2 if config.value_group_axis == "token" else 3
    if config.scale_dtype not in SCALE_DTYPE_CODE:
        raise ValueError("scale_dtype must be torch.float16, torch.bfloat16 or torch.float32.")

    def make(bits, axis, rotation, n):
        if n == 0:
            return None
        if rotation == "hadamard" and (D < 1 or D & (D - 1)):
            raise ValueError("hadamard rotation requires a power-of-two head dimension.")
        axis_len = n if axis == 2 else D
        return TensorPlan(bits=bits, quantizer=qc.quantizer, axis=axis, group_size=min(config.group_size, axis_len),
                          rotation=rotation, packed=bits in (2, 4) and config.pack_int4,
                          scale_dtype=config.scale_dtype, n=n, B=B, H=H, D=D)

    low = config.low_priority_bits or qc.bits
    return [
        make(qc.key_bits or qc.bits, key_axis, qc.rotation, tiers.n_standard),
        make(qc.value_bits or qc.bits, value_axis, qc.rotation, tiers.n_standard),
        make(config.low_priority_key_bits or low, key_axis, qc.rotation, tiers.n_cold),
        make(config.low_priority_value_bits or low, value_axis,
             effective_cold_value_rotation(config, T, qc.rotation), tiers.n_cold),
    ]


def layer_memory_bytes(shape: tuple, dtype: torch.dtype, tiers: TierSizes, plans: list) -> int:
    """Compressed bytes of one layer (core.py:194-215), computed before any kernel runs."""
    B, H, T, D = shape
    esize = torch.empty((), dtype=dtype).element_size()
    n = sum(p.memory_bytes() for p in plans if p is not None)
    n += 4 * T  # the three index lists cover every token once
    n += 2 * B * H * tiers.n_retained * D * esize
    return n
