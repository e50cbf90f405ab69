"""Compressed KV containers and the quantize / dequantize orchestration.

Mirrors the public surface of the reference's ``src/graphkv/core.py``
(``QuantizedTensor``, ``QuantizedKvLayer``, ``QuantizedKvCache``,
``quantize_kv_layer``, ``build_retention_mask``, ``hf_cache_to_tuple``, ...) with
the same field names, tensor shapes, byte layouts, statistics and exceptions.
The data path runs in the CUDA kernels of ``libgraphkv_b200.so``:

* layers of one cache that share a geometry and an importance-score tensor are
  compressed by ONE selection launch and ONE quantize launch; their outputs
  live in one device arena and each layer's tensors are views into it;
* tier sizes and byte counts are computed on the host before any kernel runs,
  so the passthrough decision (core.py:770-772) needs no device sync;
* dequantization of consecutive layers of one arena is one launch that writes
  every output row exactly once.

Inputs may live on the host: they are copied to the current CUDA device, and
the exported (dequantized) caches are returned on the input's device.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from math import sqrt
from typing import Iterable, Literal, Sequence

import torch
from torch.nn import functional as F

from . import _lib as L
from .config import (
    KvQuantConfig,
    TensorPlan,
    TierSizes,
    effective_low_priority_ratio,
    keep_count,
    layer_memory_bytes,
    resolve_tiers,
    tensor_plans,
)

_ALIGN = 256


def _tensor_nbytes(tensor: torch.Tensor | None) -> int:
    if tensor is None:
        return 0
    return tensor.numel() * tensor.element_size()


def _dtype_element_size(dtype: torch.dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


def _compute_device(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("graphkv_b200 needs a CUDA device; there is no CPU fallback.")
    return torch.device("cuda", torch.cuda.current_device())


def _to_device(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    if t.device == device:
        return t
    return t.to(device, non_blocking=t.is_pinned())


# ---------------------------------------------------------------------------
# containers
# ---------------------------------------------------------------------------

@dataclass
class QuantizedTensor:
    """One compressed tensor (core.py:130-173): packed codes ``q`` (one
    little-end-first byte stream of the moved, padded ``q_shape`` tensor),
    ``scales`` ``[..., n_groups, 1]`` and optional uint8 ``zero_points``."""

    q: torch.Tensor
    scales: torch.Tensor
    zero_points: torch.Tensor | None
    original_shape: tuple[int, ...]
    axis: int
    group_size: int
    bits: int
    padded: int
    q_shape: tuple[int, ...]
    original_dtype: torch.dtype
    packed: bool
    packed_offset: int
    rotation: str = "none"

    @property
    def qmin(self) -> int:
        return -(1 << (self.bits - 1))

    def memory_bytes(self) -> int:
        return _tensor_nbytes(self.q) + _tensor_nbytes(self.scales) + _tensor_nbytes(self.zero_points)

    def _spec(self) -> L.TensorSpec:
        return L.TensorSpec(self.bits, L.GKV_AFFINE if self.zero_points is not None else L.GKV_SYMMETRIC,
                            L.GKV_AXIS_TOKEN if self.axis == 2 else L.GKV_AXIS_CHANNEL, self.group_size,
                            L.GKV_ROT_HADAMARD if self.rotation == "hadamard" else L.GKV_ROT_NONE,
                            1 if self.packed else 0, L.DTYPE_CODE[self.scales.dtype], 0)

    def dequantize(self) -> torch.Tensor:
        """The dequantized tier tensor ``original_shape`` (core.py:153-173)."""
        lib = L.lib()
        B, H, n, D = self.original_shape
        dev = self.q.device
        plan = L.Plan()
        plan.batch, plan.head_dim, plan.seq_len = B, D, n
        plan.dtype = L.DTYPE_CODE[self.original_dtype]
        plan.n_retained, plan.n_standard, plan.n_cold = 0, n, 0
        ident = torch.arange(n, dtype=torch.int32, device=dev)
        plan.idx_standard = ident.data_ptr()
        for slot in (L.STD_K, L.STD_V):
            plan.spec[slot] = self._spec()
            plan.codes[slot] = self.q.data_ptr()
            plan.scales[slot] = self.scales.data_ptr()
            plan.zero_points[slot] = L.ptr(self.zero_points)
        plan.hadamard_divisor = sqrt(D)  # the c_float field rounds it to fp32, as torch does
        out = torch.empty((2, B, H, n, D), dtype=self.original_dtype, device=dev)
        with torch.cuda.device(dev):
            L.check(lib.gkv_dequantize(ctypes.byref(plan), B * H, out[0].data_ptr(), out[1].data_ptr(), None, 0,
                                       L.stream_handle(dev)))
        return out[0]


@dataclass
class QuantizedKvLayer:
    """One quantized layer of a transformer KV cache (core.py:176-348)."""

    compressed_keys: QuantizedTensor | None
    compressed_values: QuantizedTensor | None
    compressed_indices: torch.Tensor
    retained_keys: torch.Tensor
    retained_values: torch.Tensor
    retained_indices: torch.Tensor
    original_shape: tuple[int, ...]
    seq_dim: int = 2
    passthrough_keys: torch.Tensor | None = None
    passthrough_values: torch.Tensor | None = None
    low_priority_compressed_keys: QuantizedTensor | None = None
    low_priority_compressed_values: QuantizedTensor | None = None
    low_priority_compressed_indices: torch.Tensor | None = None
    home_device: torch.device | None = None  # device of the input tensors (outputs return there)

    def memory_bytes(self) -> int:
        if self.passthrough_keys is not None and self.passthrough_values is not None:
            return _tensor_nbytes(self.passthrough_keys) + _tensor_nbytes(self.passthrough_values)
        n = 0
        for t in (self.compressed_keys, self.compressed_values, self.low_priority_compressed_keys,
                  self.low_priority_compressed_values):
            if t is not None:
                n += t.memory_bytes()
        return (n + _tensor_nbytes(self.compressed_indices) + _tensor_nbytes(self.low_priority_compressed_indices)
                + _tensor_nbytes(self.retained_keys) + _tensor_nbytes(self.retained_values)
                + _tensor_nbytes(self.retained_indices))

    def original_memory_bytes(self) -> int:
        dtype = self.retained_keys.dtype
        if self.passthrough_keys is not None:
            dtype = self.passthrough_keys.dtype
        if self.compressed_keys is not None:
            dtype = self.compressed_keys.original_dtype
        elements = 1
        for dim in self.original_shape:
            elements *= dim
        return 2 * elements * _dtype_element_size(dtype)

    def compression_ratio(self) -> float:
        return self.original_memory_bytes() / max(self.memory_bytes(), 1)

    def stats(self) -> dict[str, float]:
        original_bytes = self.original_memory_bytes()
        compressed_bytes = self.memory_bytes()
        retained = self.retained_token_count()
        compressed = self.compressed_token_count()
        low = self.low_priority_token_count()
        total = retained + compressed
        return {
            "original_bytes": float(original_bytes),
            "compressed_bytes": float(compressed_bytes),
            "compression_ratio": original_bytes / max(compressed_bytes, 1),
            "retained_tokens": float(retained),
            "compressed_tokens": float(compressed),
            "standard_compressed_tokens": float(compressed - low),
            "low_priority_tokens": float(low),
            "retained_fraction": retained / max(total, 1),
            "compressed_fraction": compressed / max(total, 1),
        }

    def retained_token_count(self) -> int:
        if self.passthrough_keys is not None:
            return self.original_shape[self.seq_dim]
        return int(self.retained_indices.numel())

    def compressed_token_count(self) -> int:
        if self.passthrough_keys is not None:
            return 0
        return int(self.compressed_indices.numel()) + self.low_priority_token_count()

    def low_priority_token_count(self) -> int:
        if self.passthrough_keys is not None or self.low_priority_compressed_indices is None:
            return 0
        return int(self.low_priority_compressed_indices.numel())

    def dequantize(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Keys and values ``[B, H, T, D]`` (core.py:265-307), on the input's device."""
        if self.passthrough_keys is not None and self.passthrough_values is not None:
            return self.passthrough_keys, self.passthrough_values
        return _dequantize_layers([self])[0]

    def report(self, original_keys: torch.Tensor, original_values: torch.Tensor) -> dict[str, float]:
        """Bytes, token counts and reconstruction error against the original
        tensors (core.py:309-323)."""
        keys, values = self.dequantize()
        given = _tensor_nbytes(original_keys) + _tensor_nbytes(original_values)
        stored = self.memory_bytes()
        out = {"original_bytes": float(given), "quantized_bytes": float(stored),
               "compression_ratio": given / max(stored, 1),
               "retained_tokens": float(self.retained_token_count()),
               "compressed_tokens": float(self.compressed_token_count())}
        pairs = (("key", keys, original_keys.to(keys.device)), ("value", values, original_values.to(values.device)))
        for name, got, want in pairs:
            out[f"{name}_mse"] = float(F.mse_loss(got.float(), want.float()).cpu())
        for name, got, want in pairs:
            out[f"{name}_cosine"] = _flat_cosine(got, want)
        return out

    def append(self, new_keys: torch.Tensor, new_values: torch.Tensor, config: KvQuantConfig,
               importance_scores: torch.Tensor | None = None) -> "QuantizedKvLayer":
        """This layer with ``new_keys`` / ``new_values`` [B, H, n, D] appended,
        requantized as the reference does (core.py:325-348)."""
        return append_layers([self], [(new_keys, new_values)], config, importance_scores)[0]


@dataclass
class QuantizedKvCache:
    layers: list[QuantizedKvLayer]

    @classmethod
    def from_past_key_values(
        cls,
        past_key_values: Sequence[tuple[torch.Tensor, torch.Tensor]],
        config: KvQuantConfig,
        importance_scores: Sequence[torch.Tensor] | torch.Tensor | None = None,
    ) -> "QuantizedKvCache":
        """core.py:355-369, batched: one selection and one quantize launch per run
        of layers with the same geometry and scores."""
        pairs = list(past_key_values)
        per_layer = []
        for layer_idx, (keys, values) in enumerate(pairs):
            if isinstance(importance_scores, torch.Tensor) or importance_scores is None:
                per_layer.append(importance_scores)
            else:
                per_layer.append(importance_scores[layer_idx])
        return cls(_quantize_layers(pairs, config, per_layer))

    def dequantize(self) -> tuple[tuple[torch.Tensor, torch.Tensor], ...]:
        return tuple(_dequantize_layers(self.layers))

    def memory_bytes(self) -> int:
        return sum(layer.memory_bytes() for layer in self.layers)

    def original_memory_bytes(self) -> int:
        return sum(layer.original_memory_bytes() for layer in self.layers)

    def compression_ratio(self) -> float:
        return self.original_memory_bytes() / max(self.memory_bytes(), 1)

    def retained_token_count(self) -> int:
        return sum(layer.retained_token_count() for layer in self.layers)

    def compressed_token_count(self) -> int:
        return sum(layer.compressed_token_count() for layer in self.layers)

    def low_priority_token_count(self) -> int:
        return sum(layer.low_priority_token_count() for layer in self.layers)

    def stats(self) -> dict[str, float]:
        """core.py:392-413."""
        original_bytes = self.original_memory_bytes()
        compressed_bytes = self.memory_bytes()
        retained = self.retained_token_count()
        compressed = self.compressed_token_count()
        low = self.low_priority_token_count()
        total = retained + compressed
        ratios = [layer.compression_ratio() for layer in self.layers]
        return {
            "layers": float(len(self.layers)),
            "original_bytes": float(original_bytes),
            "compressed_bytes": float(compressed_bytes),
            "compression_ratio": original_bytes / max(compressed_bytes, 1),
            "retained_tokens": float(retained),
            "compressed_tokens": float(compressed),
            "standard_compressed_tokens": float(compressed - low),
            "low_priority_tokens": float(low),
            "retained_fraction": retained / max(total, 1),
            "compressed_fraction": compressed / max(total, 1),
            "min_layer_compression_ratio": min(ratios, default=0.0),
            "max_layer_compression_ratio": max(ratios, default=0.0),
        }

    def layer_stats(self) -> tuple[dict[str, float], ...]:
        return tuple(layer.stats() for layer in self.layers)

    def append(self, new_past_key_values: Sequence[tuple[torch.Tensor, torch.Tensor]], config: KvQuantConfig,
               importance_scores: Sequence[torch.Tensor] | torch.Tensor | None = None) -> "QuantizedKvCache":
        """Every layer with its new tokens appended and requantized (core.py:418-433)."""
        return QuantizedKvCache(append_layers(self.layers, new_past_key_values, config, importance_scores))

    @classmethod
    def from_hf_cache(cls, cache: object, config: KvQuantConfig,
                      importance_scores: Sequence[torch.Tensor] | torch.Tensor | None = None,
                      cache_role: Literal["self", "cross"] = "self") -> "QuantizedKvCache":
        return cls.from_past_key_values(hf_cache_to_tuple(cache, cache_role=cache_role), config, importance_scores)

    def to_legacy_cache(self) -> tuple[tuple[torch.Tensor, torch.Tensor], ...]:
        return self.dequantize()

    def to_hf_cache(self, implementation: Literal["dynamic", "static", "sliding_window", "legacy"] = "dynamic", *,
                    config: object | None = None, max_cache_len: int | None = None) -> object:
        """core.py:450-470."""
        if implementation == "legacy":
            return self.to_legacy_cache()
        if implementation == "dynamic":
            return self.to_hf_dynamic_cache(config=config)
        if implementation in {"static", "sliding_window"}:
            return self._to_hf_positioned_cache(implementation, config=config, max_cache_len=max_cache_len)
        raise ValueError("implementation must be 'dynamic', 'static', 'sliding_window', or 'legacy'.")

    def to_hf_dynamic_cache(self, *, config: object | None = None) -> object:
        """core.py:472-481."""
        return _dynamic_cache_from(self.dequantize(), config)

    def _to_hf_positioned_cache(self, implementation: Literal["static", "sliding_window"], *,
                                config: object | None, max_cache_len: int | None) -> object:
        """core.py:483-508."""
        return _positioned_cache_from(self.dequantize, implementation, config, max_cache_len)


def _dynamic_cache_from(dequantized, config: object | None) -> object:
    """DynamicCache of dequantized (K, V) pairs (core.py:472-481).  A plain
    ``DynamicLayer`` receives the tensors directly (its ``update`` would
    concatenate them onto an empty tensor, a full copy with the same result);
    other layer types go through ``update``."""
    try:
        from transformers.cache_utils import DynamicCache, DynamicLayer
    except ImportError as exc:
        raise RuntimeError("transformers is required to build a DynamicCache.") from exc
    cache = DynamicCache(config=config)
    for layer_idx, (keys, values) in enumerate(dequantized):
        if not getattr(cache, "offloading", False) and getattr(cache, "layer_class_to_replicate", None) is not None:
            while len(cache.layers) <= layer_idx:
                cache.layers.append(cache.layer_class_to_replicate())
        target = cache.layers[layer_idx] if layer_idx < len(cache.layers) else None
        if (type(target) is DynamicLayer and not getattr(target, "is_initialized", True)
                and not getattr(cache, "offloading", False)):
            target.lazy_initialization(keys, values)
            target.keys = keys
            target.values = values
        else:
            cache.update(keys, values, layer_idx)
    return cache


_POSITIONED_CACHES = {"static": "StaticCache", "sliding_window": "SlidingWindowCache"}


def _positioned_cache_from(dequantized, implementation: Literal["static", "sliding_window"],
                           config: object | None, max_cache_len: int | None) -> object:
    """Static / sliding-window HF cache of the dequantized pairs (core.py:483-508);
    ``dequantized`` is a callable, so a missing config or transformers raises
    before any dequantization."""
    if config is None:
        raise ValueError("config is required for static or sliding_window HF cache export.")
    try:
        from transformers import cache_utils
        cache_cls = getattr(cache_utils, _POSITIONED_CACHES[implementation])
    except (ImportError, AttributeError) as exc:
        raise RuntimeError("transformers is required to build a positioned cache.") from exc
    pairs = list(dequantized())
    longest = max((k.shape[2] for k, _ in pairs), default=0)
    capacity = longest if max_cache_len is None else max_cache_len
    if capacity < longest:
        raise ValueError("max_cache_len must be at least the longest KV sequence length.")
    cache = cache_cls(config, max_cache_len=capacity)
    for index, (keys, values) in enumerate(pairs):
        where = torch.arange(keys.shape[2], device=keys.device, dtype=torch.long)
        cache.update(keys, values, index, cache_kwargs={"cache_position": where})
    return cache


def export_dequantized(dequantized, implementation: str, *, config: object | None = None,
                       max_cache_len: int | None = None) -> object:
    """Dequantized (K, V) pairs in the cache format ``implementation`` (the
    dispatch of core.py:450-470)."""
    if implementation == "legacy":
        return tuple(dequantized)
    if implementation == "dynamic":
        return _dynamic_cache_from(dequantized, config)
    if implementation in {"static", "sliding_window"}:
        return _positioned_cache_from(lambda: dequantized, implementation, config, max_cache_len)
    raise ValueError("implementation must be 'dynamic', 'static', 'sliding_window', or 'legacy'.")


# ---------------------------------------------------------------------------
# HF cache extraction (core.py:511-592)
# ---------------------------------------------------------------------------

def _encoder_decoder_pairs(cache: object, role: str):
    """An encoder-decoder cache: the pairs of its self or cross attention part."""
    if not (hasattr(cache, "self_attention_cache") or hasattr(cache, "cross_attention_cache")):
        return None
    if role not in ("self", "cross"):
        raise ValueError("cache_role must be 'self' or 'cross'.")
    part = getattr(cache, f"{role}_attention_cache", None)
    if part is None:
        raise TypeError(f"HF encoder-decoder cache has no {role!r} attention cache.")
    return hf_cache_to_tuple(part)


def _legacy_pairs(cache: object, role: str):
    """A legacy tuple / list of (K, V, ...) entries; empty entries are skipped."""
    if not isinstance(cache, (tuple, list)):
        return None
    pairs = []
    for entry in cache:
        if entry is None:
            continue
        if not isinstance(entry, (tuple, list)) or len(entry) < 2:
            raise TypeError("Legacy cache layers must be tuples/lists with at least key and value tensors.")
        if entry[0] is not None and entry[1] is not None:
            pairs.append((entry[0], entry[1]))
    return tuple(pairs)


def _reported_length(layer: object):
    """Filled length a cache layer reports: get_seq_length(), else cumulative_length."""
    get_length = getattr(layer, "get_seq_length", None)
    if callable(get_length):
        try:
            n = get_length()
        except TypeError:
            n = None
        if n is not None:
            return n
    return getattr(layer, "cumulative_length", None)


def _filled_length(layer: object, keys: torch.Tensor) -> int:
    """Tokens of a cache layer that hold data: a dynamic layer is full; a layer
    with preallocated storage (static / sliding) reports its filled length."""
    capacity = keys.shape[2]
    if "dynamic" in type(layer).__name__.lower():
        return capacity
    n = _reported_length(layer)
    if n is None:
        return capacity
    if isinstance(n, torch.Tensor):
        n = int(n.max().item()) if n.numel() else 0
    return min(max(int(n), 0), capacity)


def _layered_pairs(cache: object, role: str):
    """A cache with ``.layers`` (transformers >= 4.56): each layer's filled prefix."""
    layers = getattr(cache, "layers", None)
    if layers is None:
        return None
    pairs = []
    for layer in layers:
        keys, values = getattr(layer, "keys", None), getattr(layer, "values", None)
        if keys is None or values is None:
            continue
        n = _filled_length(layer, keys)
        if n == 0:
            continue
        if n < keys.shape[2]:
            keys, values = keys[:, :, :n].contiguous(), values[:, :, :n].contiguous()
        pairs.append((keys, values))
    return tuple(pairs)


def _split_lists_pairs(cache: object, role: str):
    """A cache with parallel ``key_cache`` / ``value_cache`` lists."""
    key_list, value_list = getattr(cache, "key_cache", None), getattr(cache, "value_cache", None)
    if key_list is None or value_list is None:
        return None
    return tuple((k, v) for k, v in zip(key_list, value_list) if k is not None and v is not None)


_CACHE_READERS = (_encoder_decoder_pairs, _legacy_pairs, _layered_pairs, _split_lists_pairs)


def hf_cache_to_tuple(cache: object, *, cache_role: Literal["self", "cross"] = "self"
                      ) -> tuple[tuple[torch.Tensor, torch.Tensor], ...]:
    """(keys, values) pairs of a legacy or Hugging Face cache (core.py:511-592):
    the first reader that recognises the cache's form decides."""
    for read in _CACHE_READERS:
        pairs = read(cache, cache_role)
        if pairs is not None:
            return pairs
    raise TypeError(f"Unsupported cache type: {type(cache)!r}")


# ---------------------------------------------------------------------------
# selection helpers with the reference's signatures
# ---------------------------------------------------------------------------

def _sum_last_block(rows: int, cols: int, threads: int) -> int:
    """First column of the last per-thread column block of torch's CPU reduction
    of a contiguous [rows, cols] tensor over rows: at::parallel_for splits the
    columns into ceil(cols / threads)-wide blocks whose ends are rounded down to
    32 columns (the last end excepted); small reductions (fewer than 32768
    elements) and single-threaded runs form one block."""
    if rows * cols < 32768 or threads <= 1 or cols <= 1:
        return 0
    nt = min(threads, cols)
    width = -(-cols // nt)
    last = 0
    for tid in range(nt):
        begin = tid * width
        if begin >= cols:
            break
        end = min(cols, begin + width)
        begin -= begin % 32
        if end != cols:
            end -= end % 32
        if begin < end:
            last = begin
    return last


def _normalize_token_scores(seq_len: int, scores: torch.Tensor, device: torch.device) -> torch.Tensor:
    """fp32 [T] scores on ``device`` (core.py:1019-1031).  Multi-dimensional
    scores are averaged by ``gkv_mean_scores`` in the fp32 addition order of
    torch's CPU mean for this process's thread count, so the means -- and the
    selections that depend on their last bit -- are those of the reference run
    on the CPU."""
    scores = scores.to(device=device, dtype=torch.float32)
    if scores.numel() == seq_len:
        return scores.reshape(seq_len)
    if scores.ndim >= 1 and scores.shape[-1] == seq_len:
        x, axis, n_out = scores.reshape(-1, seq_len).contiguous(), 0, seq_len
    elif scores.ndim >= 1 and scores.shape[0] == seq_len:
        x, axis, n_out = scores.reshape(seq_len, -1).contiguous(), 1, seq_len
    else:
        raise ValueError("importance_scores must have one score per token or a final token dimension.")
    rows, cols = x.shape
    last = _sum_last_block(rows, cols, torch.get_num_threads()) if axis == 0 else 0
    out = torch.empty(n_out, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        L.check(L.lib().gkv_mean_scores(x.data_ptr(), rows, cols, axis, last, out.data_ptr(),
                                        L.stream_handle(device)))
    return out


def _select(T: int, config: KvQuantConfig, scores: torch.Tensor | None, device: torch.device,
            outlier: torch.Tensor | None = None, tiers: TierSizes | None = None):
    """Run the selection kernel; returns (tiers, idx_ret, idx_std, idx_cold) int32 device tensors."""
    lib = L.lib()
    tiers = tiers or resolve_tiers(config, T, scores is not None)
    s = None
    if scores is not None:
        s = _normalize_token_scores(T, scores, device).contiguous()
    idx = torch.empty(T, dtype=torch.int32, device=device)
    idx_ret, idx_std, idx_cold = torch.split(idx, [tiers.n_retained, tiers.n_standard, tiers.n_cold])
    ws = torch.empty(max(int(lib.gkv_select_workspace_bytes(T)), 1), dtype=torch.uint8, device=device)
    pol = tiers.policy()
    with torch.cuda.device(device):
        L.check(lib.gkv_select_tiers(L.ptr(s), L.ptr(outlier), ctypes.byref(pol), idx_ret.data_ptr(),
                                     idx_std.data_ptr(), idx_cold.data_ptr(), ws.data_ptr(), ws.numel(),
                                     L.stream_handle(device)))
    return tiers, idx_ret, idx_std, idx_cold


def build_retention_mask(seq_len: int, config: KvQuantConfig, importance_scores: torch.Tensor | None = None,
                         device: torch.device | None = None) -> torch.Tensor:
    """Token mask for full-precision retention (core.py:595-644): sink, tail and
    top importance scores, computed by the selection kernel."""
    config.validate()
    if device is None:
        device = importance_scores.device if importance_scores is not None else torch.device("cpu")
    device = torch.device(device)
    cdev = device if device.type == "cuda" else _compute_device(torch.empty(0))
    no_outlier = KvQuantConfig(**{**config.__dict__, "outlier_protection_ratio": 0.0, "min_outlier_tokens": 0,
                                  "low_priority_ratio": 0.0, "long_low_priority_ratio": None,
                                  "min_low_priority_tokens": 0})
    _, idx_ret, _, _ = _select(seq_len, no_outlier, importance_scores, cdev)
    mask = torch.zeros(seq_len, dtype=torch.bool, device=cdev)
    mask[idx_ret.long()] = True
    return mask.to(device)


def chunk_scores_to_token_scores(seq_len: int, chunk_spans: Iterable[tuple[int, int]], chunk_scores: torch.Tensor,
                                 device: torch.device | None = None) -> torch.Tensor:
    """Spread chunk-level scores over token positions (core.py:775-797): max over
    the covering chunks, 0 for uncovered tokens."""
    if device is None:
        device = chunk_scores.device
    token_scores = torch.full((seq_len,), -torch.inf, dtype=torch.float32, device=device)
    scores = chunk_scores.to(device=device, dtype=torch.float32).flatten()
    for idx, (start, end) in enumerate(chunk_spans):
        if idx >= scores.numel():
            break
        lo, hi = max(0, int(start)), min(seq_len, int(end))
        if hi <= lo:
            continue
        token_scores[lo:hi] = torch.maximum(token_scores[lo:hi], scores[idx])
    return torch.nan_to_num(token_scores, neginf=0.0)


# ---------------------------------------------------------------------------
# quantize orchestration
# ---------------------------------------------------------------------------

def _check_pair(keys: torch.Tensor, values: torch.Tensor) -> None:
    if keys.shape != values.shape:
        raise ValueError("keys and values must have the same shape.")
    if keys.ndim != 4:
        raise ValueError("keys and values must use [batch, heads, tokens, head_dim] layout.")
    if keys.dtype not in L.DTYPE_CODE or values.dtype != keys.dtype:
        raise ValueError("keys and values must be float32, float16 or bfloat16 tensors of one dtype.")


def _full_precision_layer(keys: torch.Tensor, values: torch.Tensor, seq_dim: int = 2) -> QuantizedKvLayer:
    """core.py:959-976."""
    empty_indices = torch.empty(0, dtype=torch.int32, device=keys.device)
    shape = list(keys.shape)
    shape[seq_dim] = 0
    return QuantizedKvLayer(compressed_keys=None, compressed_values=None, compressed_indices=empty_indices,
                            retained_keys=keys.new_empty(tuple(shape)), retained_values=values.new_empty(tuple(shape)),
                            retained_indices=empty_indices, original_shape=tuple(keys.shape), seq_dim=seq_dim,
                            passthrough_keys=keys.detach().contiguous(),
                            passthrough_values=values.detach().contiguous(), home_device=keys.device)


class _Arena:
    """One uint8 device allocation carved into 256-byte aligned regions."""

    def __init__(self):
        self.sizes = []

    def reserve(self, nbytes: int) -> int:
        self.sizes.append(nbytes)
        return len(self.sizes) - 1

    def allocate(self, device: torch.device):
        offs, off = [], 0
        for n in self.sizes:
            offs.append(off)
            off += (n + _ALIGN - 1) // _ALIGN * _ALIGN
        self.buf = torch.empty(max(off, 1), dtype=torch.uint8, device=device)
        self.offs = offs

    def view(self, handle: int, start: int, nbytes: int, dtype: torch.dtype, shape: tuple) -> torch.Tensor:
        o = self.offs[handle] + start
        return self.buf.narrow(0, o, nbytes).view(dtype).view(shape)

    def ptr(self, handle: int) -> int:
        return self.buf.data_ptr() + self.offs[handle]


def _quantize_layers(pairs, config: KvQuantConfig, per_layer_scores) -> list[QuantizedKvLayer]:
    config.validate()
    for keys, values in pairs:
        _check_pair(keys, values)
    out: list[QuantizedKvLayer] = []
    i = 0
    while i < len(pairs):
        k0 = pairs[i][0]
        s0 = per_layer_scores[i]
        j = i + 1
        while (j < len(pairs) and pairs[j][0].shape == k0.shape and pairs[j][0].dtype == k0.dtype
               and pairs[j][0].device == k0.device and per_layer_scores[j] is s0):
            j += 1
        out.extend(_quantize_group(pairs[i:j], config, s0))
        i = j
    return out


def _layer_input(keys: torch.Tensor, values: torch.Tensor) -> L.LayerIn:
    li = L.LayerIn()
    li.k, li.v = keys.data_ptr(), values.data_ptr()
    for q in range(3):
        li.k_stride[q] = keys.stride(q)
        li.v_stride[q] = values.stride(q)
    li.heads = keys.shape[1]
    return li


class _GroupRun:
    """Compression of a run of layers of one geometry sharing one selection:
    device arena for every stored tensor, the C plan, the layer inputs and the
    workspaces, built once.  ``select()`` / ``quantize()`` / ``dequantize()``
    only launch kernels, so a prepared run can be executed repeatedly."""

    def __init__(self, dev_pairs, config: KvQuantConfig, tiers: TierSizes, plans: list, device: torch.device,
                 home: torch.device, idx=None):
        lib = L.lib()
        k0 = dev_pairs[0][0]
        B, H, T, D = k0.shape
        dtype = k0.dtype
        self.device, self.home, self.dtype, self.shape = device, home, dtype, (B, H, T, D)
        self.pairs, self.tiers, self.plans, self.config = dev_pairs, tiers, plans, config
        nl = len(dev_pairs)
        esize = _dtype_element_size(dtype)
        ar = _Arena()
        h_idx = ar.reserve(4 * T) if idx is None else None
        h_ret = [ar.reserve(nl * B * H * tiers.n_retained * D * esize) for _ in range(2)]
        h_codes, h_scales, h_zps = [None] * 4, [None] * 4, [None] * 4
        for i, p in enumerate(plans):
            if p is None:
                continue
            h_codes[i] = ar.reserve(nl * p.code_bytes)
            h_scales[i] = ar.reserve(nl * p.n_groups * _dtype_element_size(p.scale_dtype))
            if p.quantizer == "affine":
                h_zps[i] = ar.reserve(nl * p.n_groups)
        ar.allocate(device)
        self.arena, self.h_ret, self.h_codes, self.h_scales, self.h_zps = ar, h_ret, h_codes, h_scales, h_zps
        if idx is None:
            all_idx = ar.view(h_idx, 0, 4 * T, torch.int32, (T,))
            idx = torch.split(all_idx, [tiers.n_retained, tiers.n_standard, tiers.n_cold])
        self.idx_ret, self.idx_std, self.idx_cold = idx

        plan = L.Plan()
        plan.batch, plan.head_dim, plan.seq_len, plan.dtype = B, D, T, L.DTYPE_CODE[dtype]
        plan.n_retained, plan.n_standard, plan.n_cold = tiers.n_retained, tiers.n_standard, tiers.n_cold
        plan.idx_retained = self.idx_ret.data_ptr()
        plan.idx_standard = self.idx_std.data_ptr()
        plan.idx_cold = self.idx_cold.data_ptr()
        plan.hadamard_divisor = sqrt(D)  # the c_float field rounds it to fp32, as torch does
        plan.retained_k, plan.retained_v = ar.ptr(h_ret[0]), ar.ptr(h_ret[1])
        for i, p in enumerate(plans):
            if p is None:
                continue
            plan.spec[i] = p.spec()
            plan.codes[i] = ar.ptr(h_codes[i])
            plan.scales[i] = ar.ptr(h_scales[i])
            plan.zero_points[i] = ar.ptr(h_zps[i]) if h_zps[i] is not None else 0
        self.plan = plan
        self.layer_ins = (L.LayerIn * nl)(*[_layer_input(k, v) for k, v in dev_pairs])
        ws_bytes = int(lib.gkv_quantize_workspace_bytes(ctypes.byref(plan), self.layer_ins, nl))
        self.ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
        self.ws_bytes = ws_bytes
        self.sel_ws = torch.empty(max(int(lib.gkv_select_workspace_bytes(T)), 1), dtype=torch.uint8, device=device)
        self.policy = tiers.policy()
        self.outlier = torch.empty(T, dtype=torch.float32, device=device) if tiers.keep_outlier > 0 else None
        self.out_k = self.out_v = None

    def select(self, scores: torch.Tensor | None) -> None:
        """Selection kernel(s) for normalized fp32 [T] scores on the device."""
        lib = L.lib()
        st = L.stream_handle(self.device)
        with torch.cuda.device(self.device):
            if self.outlier is not None:
                li = self.layer_ins[0]
                B, _, T, D = self.shape
                L.check(lib.gkv_outlier_scores(ctypes.byref(li), B, T, D, L.DTYPE_CODE[self.dtype],
                                               self.outlier.data_ptr(), st))
            L.check(lib.gkv_select_tiers(L.ptr(scores), L.ptr(self.outlier), ctypes.byref(self.policy),
                                         self.idx_ret.data_ptr(), self.idx_std.data_ptr(), self.idx_cold.data_ptr(),
                                         self.sel_ws.data_ptr(), self.sel_ws.numel(), st))

    def quantize(self) -> None:
        with torch.cuda.device(self.device):
            L.check(L.lib().gkv_quantize(ctypes.byref(self.plan), self.layer_ins, len(self.pairs),
                                         self.ws.data_ptr(), self.ws_bytes, L.stream_handle(self.device)))

    def dequantize(self) -> None:
        """Dequantize every layer of the run into preallocated [L, B, H, T, D] outputs."""
        if self.out_k is None:
            shp = (len(self.pairs), *self.shape)
            self.out_k = torch.empty(shp, dtype=self.dtype, device=self.device)
            self.out_v = torch.empty(shp, dtype=self.dtype, device=self.device)
        B, H = self.shape[:2]
        with torch.cuda.device(self.device):
            L.check(L.lib().gkv_dequantize(ctypes.byref(self.plan), len(self.pairs) * B * H, self.out_k.data_ptr(),
                                           self.out_v.data_ptr(), None, 0, L.stream_handle(self.device)))

    def layers(self) -> list:
        """QuantizedKvLayer objects whose tensors are views into the arena."""
        B, H, T, D = self.shape
        dtype, ar, tiers = self.dtype, self.arena, self.tiers
        esize = _dtype_element_size(dtype)
        out = []
        ret_shape = (B, H, tiers.n_retained, D)
        ret_bytes = B * H * tiers.n_retained * D * esize
        for l in range(len(self.pairs)):
            qts = []
            for i, p in enumerate(self.plans):
                if p is None:
                    qts.append(None)
                    continue
                ssize = _dtype_element_size(p.scale_dtype)
                q_dtype = torch.uint8 if (p.packed or p.quantizer == "affine") else torch.int8
                q_shape_store = (p.code_bytes,) if p.packed else p.q_shape
                q = ar.view(self.h_codes[i], l * p.code_bytes, p.code_bytes, q_dtype, q_shape_store)
                sc = ar.view(self.h_scales[i], l * p.n_groups * ssize, p.n_groups * ssize, p.scale_dtype,
                             p.scales_shape)
                zp = None
                if self.h_zps[i] is not None:
                    zp = ar.view(self.h_zps[i], l * p.n_groups, p.n_groups, torch.uint8, p.scales_shape)
                qts.append(QuantizedTensor(q=q, scales=sc, zero_points=zp, original_shape=(B, H, p.n, D),
                                           axis=p.axis, group_size=p.group_size, bits=p.bits, padded=p.padded,
                                           q_shape=p.q_shape, original_dtype=dtype, packed=p.packed,
                                           packed_offset=0 if p.quantizer == "affine" else -(1 << (p.bits - 1)),
                                           rotation=p.rotation))
            out.append(QuantizedKvLayer(
                compressed_keys=qts[0], compressed_values=qts[1], compressed_indices=self.idx_std,
                retained_keys=ar.view(self.h_ret[0], l * ret_bytes, ret_bytes, dtype, ret_shape),
                retained_values=ar.view(self.h_ret[1], l * ret_bytes, ret_bytes, dtype, ret_shape),
                retained_indices=self.idx_ret, original_shape=(B, H, T, D), seq_dim=2,
                low_priority_compressed_keys=qts[2], low_priority_compressed_values=qts[3],
                low_priority_compressed_indices=self.idx_cold, home_device=self.home))
        return out


def _prepare_group(pairs, config: KvQuantConfig, scores, retain_mask: torch.Tensor | None = None):
    """Split a run of same-geometry layers into prepared _GroupRun objects (or
    passthrough layers).  Returns a list of ("run", run, scores) / ("pass", layer)."""
    k0 = pairs[0][0]
    shape = tuple(k0.shape)
    B, H, T, D = shape
    dtype = k0.dtype
    home = k0.device
    device = _compute_device(k0)
    outlier_needed = config.outlier_protection_ratio > 0.0 or config.min_outlier_tokens > 0
    if retain_mask is None and outlier_needed and len(pairs) > 1:
        # outlier scores differ per layer, so each layer has its own selection
        return [item for p in pairs for item in _prepare_group([p], config, scores)]
    dev_pairs = []
    for keys, values in pairs:
        keys = _to_device(keys.detach(), device)
        values = _to_device(values.detach(), device)
        if keys.stride(3) != 1:
            keys = keys.contiguous()
        if values.stride(3) != 1:
            values = values.contiguous()
        dev_pairs.append((keys, values))
    idx = None
    if retain_mask is not None:
        tiers, *idx = _tiers_from_mask(retain_mask, T, config, scores, device)
    else:
        tiers = resolve_tiers(config, T, scores is not None)
    plans = tensor_plans(config, shape, tiers)
    if config.skip_if_not_smaller and \
            layer_memory_bytes(shape, dtype, tiers, plans) >= 2 * B * H * T * D * _dtype_element_size(dtype):
        return [("pass", _full_precision_layer(k.detach(), v.detach())) for k, v in pairs]
    if len(pairs) > 1 and any(p is not None and not p.slice_bits_aligned for p in plans):
        return [item for p in pairs for item in _prepare_group([p], config, scores)]
    s = _normalize_token_scores(T, scores, device).contiguous() if (scores is not None and idx is None) else None
    return [("run", _GroupRun(dev_pairs, config, tiers, plans, device, home, idx), s, idx is None)]


def _quantize_group(pairs, config: KvQuantConfig, scores, retain_mask: torch.Tensor | None = None
                    ) -> list[QuantizedKvLayer]:
    """Compress layers of one geometry sharing one scores tensor."""
    out = []
    for item in _prepare_group(pairs, config, scores, retain_mask):
        if item[0] == "pass":
            out.append(item[1])
            continue
        _, run, s, needs_select = item
        if needs_select:
            run.select(s)
        run.quantize()
        out.extend(run.layers())
    return out


def _tiers_from_mask(retain_mask: torch.Tensor, T: int, config: KvQuantConfig, scores, device):
    """Tiers of a caller-supplied retention mask (core.py:680-719).  The cold tier
    among the remaining tokens follows the same rule as the selection kernel
    (smallest scores, lower position first among equals)."""
    mask = retain_mask.to(device=device, dtype=torch.bool)
    if mask.numel() != T:
        raise ValueError("retain_mask must have one value per token.")
    mask = mask.reshape(T)
    positions = torch.arange(T, device=device, dtype=torch.int32)
    cold = torch.zeros(T, dtype=torch.bool, device=device)
    compressed = ~mask
    n_comp = int(compressed.sum().item())
    ratio = effective_low_priority_ratio(config, T)
    if (scores is not None and T >= config.low_priority_min_context
            and (ratio > 0.0 or config.min_low_priority_tokens > 0)
            and (config.low_priority_bits is not None or config.low_priority_key_bits is not None
                 or config.low_priority_value_bits is not None) and n_comp > 0):
        keep = keep_count(n_comp, ratio, config.min_low_priority_tokens)
        if keep > 0:
            s = _normalize_token_scores(T, scores, device)
            cand = positions[compressed]
            order = torch.sort(s[cand.long()], stable=True).indices[:keep]
            cold[cand[order].long()] = True
    standard = compressed & ~cold
    idx_ret, idx_std, idx_cold = positions[mask], positions[standard], positions[cold]
    n_ret, n_std, n_cold = idx_ret.numel(), idx_std.numel(), idx_cold.numel()
    tiers = TierSizes(T, 0, 0, 0, 0, n_cold, n_ret, n_std, n_cold)
    return tiers, idx_ret.contiguous(), idx_std.contiguous(), idx_cold.contiguous()


def quantize_kv_layer(keys: torch.Tensor, values: torch.Tensor, config: KvQuantConfig,
                      importance_scores: torch.Tensor | None = None,
                      retain_mask: torch.Tensor | None = None) -> QuantizedKvLayer:
    """Quantize one layer of KV tensors with layout [B, H, T, D] (core.py:647-772)."""
    config.validate()
    _check_pair(keys, values)
    return _quantize_group([(keys, values)], config, importance_scores, retain_mask=retain_mask)[0]


# ---------------------------------------------------------------------------
# dequantize orchestration
# ---------------------------------------------------------------------------

def _layer_tensors(layer: QuantizedKvLayer):
    return (layer.compressed_keys, layer.compressed_values, layer.low_priority_compressed_keys,
            layer.low_priority_compressed_values)


def _storage_list(layer: QuantizedKvLayer):
    out = [layer.retained_keys, layer.retained_values]
    for t in _layer_tensors(layer):
        if t is not None:
            out.extend([t.q, t.scales] + ([t.zero_points] if t.zero_points is not None else []))
    return out


def _signature(layer: QuantizedKvLayer):
    specs = tuple(None if t is None else (bytes(t._spec()), t.q.dtype, t.q_shape) for t in _layer_tensors(layer))
    lp = layer.low_priority_compressed_indices
    return (layer.original_shape, layer.retained_keys.dtype, layer.retained_keys.device, specs,
            layer.retained_indices.data_ptr(), layer.compressed_indices.data_ptr(),
            lp.data_ptr() if lp is not None else 0, layer.home_device)


def _follows(a: QuantizedKvLayer, b: QuantizedKvLayer) -> bool:
    """True when b's storage directly follows a's in every region (same arena run)."""
    if _signature(a) != _signature(b):
        return False
    for x, y in zip(_storage_list(a), _storage_list(b)):
        if not (x.is_contiguous() and y.is_contiguous()) or y.data_ptr() != x.data_ptr() + _tensor_nbytes(x):
            return False
    return True


def _dequantize_layers(layers: list[QuantizedKvLayer]) -> list:
    out = []
    host_copies = set()  # GPUs whose results are being copied into host memory
    i = 0
    while i < len(layers):
        lay = layers[i]
        if lay.passthrough_keys is not None and lay.passthrough_values is not None:
            out.append((lay.passthrough_keys, lay.passthrough_values))
            i += 1
            continue
        j = i + 1
        while j < len(layers) and layers[j].passthrough_keys is None and _follows(layers[j - 1], layers[j]):
            j += 1
        for k, v, dev in _dequantize_run(layers[i:j]):
            if k.device.type == "cpu":
                host_copies.add(dev)
            out.append((k, v))
        i = j
    for dev in host_copies:
        torch.cuda.synchronize(dev)
    return out


def _run_plan(run: list[QuantizedKvLayer]):
    """The C plan of consecutive layers of one arena; returns (plan, shape, dtype, device)."""
    first = run[0]
    B, H, T, D = first.original_shape
    qts = _layer_tensors(first)
    ref = next((t for t in qts if t is not None), None)
    dtype = ref.original_dtype if ref is not None else first.retained_keys.dtype
    dev = ref.q.device if ref is not None else first.retained_keys.device
    plan = L.Plan()
    plan.batch, plan.head_dim, plan.seq_len, plan.dtype = B, D, T, L.DTYPE_CODE[dtype]
    lp = first.low_priority_compressed_indices
    plan.n_retained = first.retained_indices.numel()
    plan.n_standard = first.compressed_indices.numel()
    plan.n_cold = lp.numel() if lp is not None else 0
    plan.idx_retained = first.retained_indices.data_ptr()
    plan.idx_standard = first.compressed_indices.data_ptr()
    plan.idx_cold = lp.data_ptr() if lp is not None else 0
    plan.hadamard_divisor = sqrt(D)  # the c_float field rounds it to fp32, as torch does
    plan.retained_k, plan.retained_v = first.retained_keys.data_ptr(), first.retained_values.data_ptr()
    for i, t in enumerate(qts):
        if t is None:
            continue
        plan.spec[i] = t._spec()
        plan.codes[i] = t.q.data_ptr()
        plan.scales[i] = t.scales.data_ptr()
        plan.zero_points[i] = L.ptr(t.zero_points)
    return plan, (B, H, T, D), dtype, dev


def _dequantize_run_into(run: list[QuantizedKvLayer], outk: torch.Tensor, outv: torch.Tensor) -> None:
    """Dequantize consecutive layers of one arena into the first T tokens of each
    slice of ``outk`` / ``outv`` [L, B, H, T', D] (T' >= T, contiguous, on the
    storage device): one launch, every output row written once."""
    plan, (B, H, T, D), _, dev = _run_plan(run)
    plan.out_seq_stride = outk.shape[3] if outk.shape[3] != T else 0
    with torch.cuda.device(dev):
        L.check(L.lib().gkv_dequantize(ctypes.byref(plan), len(run) * B * H, outk.data_ptr(), outv.data_ptr(),
                                       None, 0, L.stream_handle(dev)))


def _dequantize_run(run: list[QuantizedKvLayer]) -> list:
    """One launch for consecutive layers of one arena; returns [(K, V, device), ...]."""
    _, (B, H, T, D), dtype, dev = _run_plan(run)
    nl = len(run)
    outk = torch.empty((nl, B, H, T, D), dtype=dtype, device=dev)
    outv = torch.empty((nl, B, H, T, D), dtype=dtype, device=dev)
    _dequantize_run_into(run, outk, outv)
    home = run[0].home_device
    if home is not None and home.type == "cpu":
        hk = torch.empty(outk.shape, dtype=dtype, pin_memory=True)
        hv = torch.empty(outv.shape, dtype=dtype, pin_memory=True)
        hk.copy_(outk, non_blocking=True)
        hv.copy_(outv, non_blocking=True)
        outk, outv = hk, hv
    return [(outk[l], outv[l], dev) for l in range(nl)]


def _check_append(layer: QuantizedKvLayer, new_keys: torch.Tensor, new_values: torch.Tensor) -> None:
    old = tuple(layer.original_shape)
    if old[:2] != tuple(new_keys.shape[:2]):
        raise ValueError("new_keys batch/head dimensions must match the cached layer.")
    if old[3:] != tuple(new_keys.shape[3:]):
        raise ValueError("new_keys head_dim dimensions must match the cached layer.")
    if new_keys.shape != new_values.shape:
        raise ValueError("new_keys and new_values must have the same shape.")


def _grown_pairs(layers: list[QuantizedKvLayer], new_pairs: list) -> list:
    """(K, V) of every layer with its new tokens behind the old ones -- the
    reference's ``cat(dequantize(old), new)`` (core.py:325-348).  Consecutive
    layers of one arena with equally long appends are dequantized by one launch
    straight into the grown [L, B, H, T + n, D] buffers, so no separate
    concatenation pass runs."""
    grown: list = [None] * len(layers)
    i = 0
    while i < len(layers):
        lay = layers[i]
        nk, nv = new_pairs[i]
        if lay.passthrough_keys is not None and lay.passthrough_values is not None:
            ok, ov = lay.passthrough_keys, lay.passthrough_values
            grown[i] = (torch.cat([ok, nk.to(ok.device)], dim=2), torch.cat([ov, nv.to(ov.device)], dim=2))
            i += 1
            continue
        j = i + 1
        while (j < len(layers) and layers[j].passthrough_keys is None and _follows(layers[j - 1], layers[j])
               and new_pairs[j][0].shape == nk.shape):
            j += 1
        run = layers[i:j]
        _, (B, H, T, D), dtype, dev = _run_plan(run)
        n = nk.shape[2]
        outk = torch.empty((j - i, B, H, T + n, D), dtype=dtype, device=dev)
        outv = torch.empty((j - i, B, H, T + n, D), dtype=dtype, device=dev)
        _dequantize_run_into(run, outk, outv)
        for l in range(j - i):
            outk[l, :, :, T:].copy_(new_pairs[i + l][0])
            outv[l, :, :, T:].copy_(new_pairs[i + l][1])
        for l in range(j - i):
            grown[i + l] = (outk[l], outv[l])
        i = j
    return grown


def append_layers(layers: list[QuantizedKvLayer], new_pairs, config: KvQuantConfig,
                  importance_scores=None) -> list[QuantizedKvLayer]:
    """Append new tokens to compressed layers and requantize (core.py:325-348,
    418-433) with the result of the reference: its dequantized old tokens and
    the new ones are requantized together, since every quantization group along
    the tokens and every tier boundary can move when the cache grows.  The
    dequantized old tokens go straight into the grown device buffers, and the
    requantization is the batched quantize of ``from_past_key_values``.  The
    layers keep the device their inputs came from."""
    new_pairs = list(new_pairs)
    if len(new_pairs) != len(layers):
        raise ValueError("new_past_key_values must have one (key, value) pair per cached layer.")
    for lay, (nk, nv) in zip(layers, new_pairs):
        _check_append(lay, nk, nv)
    grown = _grown_pairs(list(layers), new_pairs)
    per_layer = [importance_scores if (importance_scores is None or isinstance(importance_scores, torch.Tensor))
                 else importance_scores[i] for i in range(len(grown))]
    out = _quantize_layers(grown, config, per_layer)
    for old, new in zip(layers, out):
        if old.home_device is not None and old.home_device.type == "cpu":
            new.home_device = old.home_device
    return out


HOST_CHUNK_BYTES = 64 << 20  # K+V bytes per stage of the pipelined host round trip (at least one layer)


def roundtrip_host_cache(pairs, config: KvQuantConfig, importance_scores=None, chunk_layers: int | None = None):
    """Compress and dequantize a cache held in pinned host memory, pipelined over
    chunks of layers on three streams: the host-to-device copy of chunk c + 1,
    the selection / quantize / dequantize kernels of chunk c and the
    device-to-host copy of chunk c - 1 overlap (both copy directions at once).
    The kernels and their outputs are those of ``from_past_key_values`` followed
    by ``dequantize``; the selection runs once and its index lists serve every
    chunk.  Returns the dequantized (K, V) pairs in pinned host memory, or None
    when the cache does not take this path (device or pageable tensors, mixed
    geometries, per-layer scores or per-layer outlier selections, passthrough
    layers); the caller then compresses and dequantizes in two steps."""
    pairs = list(pairs)
    if not pairs or not torch.cuda.is_available():
        return None
    config.validate()
    for keys, values in pairs:
        _check_pair(keys, values)
    k0 = pairs[0][0]
    shape, dtype = tuple(k0.shape), k0.dtype
    for keys, values in pairs:
        if (tuple(keys.shape) != shape or keys.dtype != dtype or keys.device.type != "cpu"
                or values.device.type != "cpu" or not keys.is_pinned() or not values.is_pinned()
                or keys.stride(3) != 1 or values.stride(3) != 1):
            return None
    if importance_scores is not None and not isinstance(importance_scores, torch.Tensor):
        return None
    if config.outlier_protection_ratio > 0.0 or config.min_outlier_tokens > 0:
        return None
    B, H, T, D = shape
    tiers = resolve_tiers(config, T, importance_scores is not None)
    plans = tensor_plans(config, shape, tiers)
    if config.skip_if_not_smaller and \
            layer_memory_bytes(shape, dtype, tiers, plans) >= 2 * B * H * T * D * _dtype_element_size(dtype):
        return None
    n = len(pairs)
    if chunk_layers is None:
        chunk_layers = -(-HOST_CHUNK_BYTES // (2 * B * H * T * D * _dtype_element_size(dtype)))
    step = max(1, min(int(chunk_layers), n))
    if step > 1 and any(p is not None and not p.slice_bits_aligned for p in plans):
        step = 1
    dev = _compute_device(torch.empty(0))
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    chunks = [(a, min(n, a + step)) for a in range(0, n, step)]
    slots = min(2, len(chunks))
    in_k = [torch.empty((step, *shape), dtype=dtype, device=dev) for _ in range(slots)]
    in_v = [torch.empty((step, *shape), dtype=dtype, device=dev) for _ in range(slots)]
    out_k = [torch.empty((step, *shape), dtype=dtype, device=dev) for _ in range(slots)]
    out_v = [torch.empty((step, *shape), dtype=dtype, device=dev) for _ in range(slots)]
    host_k = torch.empty((n, *shape), dtype=dtype, pin_memory=True)
    host_v = torch.empty((n, *shape), dtype=dtype, pin_memory=True)
    scores = None
    if importance_scores is not None:
        scores = _normalize_token_scores(T, importance_scores, dev).contiguous()
    s_in.wait_stream(comp)  # the buffers above may reuse memory of earlier work on this stream
    s_out.wait_stream(comp)
    in_free: list = [None] * slots
    out_free: list = [None] * slots
    first = None
    for c, (a, b) in enumerate(chunks):
        slot, nl = c % slots, b - a
        with torch.cuda.stream(s_in):
            if in_free[slot] is not None:
                s_in.wait_event(in_free[slot])
            for i in range(nl):
                in_k[slot][i].copy_(pairs[a + i][0], non_blocking=True)
                in_v[slot][i].copy_(pairs[a + i][1], non_blocking=True)
            loaded = torch.cuda.Event()
            loaded.record(s_in)
        comp.wait_event(loaded)
        idx = None if first is None else (first.idx_ret, first.idx_std, first.idx_cold)
        run = _GroupRun([(in_k[slot][i], in_v[slot][i]) for i in range(nl)], config, tiers, plans, dev,
                        torch.device("cpu"), idx)
        if first is None:
            run.select(scores)
            first = run
        run.quantize()
        in_free[slot] = torch.cuda.Event()
        in_free[slot].record(comp)
        if out_free[slot] is not None:
            comp.wait_event(out_free[slot])
        run.out_k, run.out_v = out_k[slot][:nl], out_v[slot][:nl]
        run.dequantize()
        decoded = torch.cuda.Event()
        decoded.record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(decoded)
            host_k[a:b].copy_(out_k[slot][:nl], non_blocking=True)
            host_v[a:b].copy_(out_v[slot][:nl], non_blocking=True)
            out_free[slot] = torch.cuda.Event()
            out_free[slot].record(s_out)
    s_out.synchronize()
    return [(host_k[l], host_v[l]) for l in range(n)]


# ---------------------------------------------------------------------------
# diagnostics (core.py:800-845, 1010-1012)
# ---------------------------------------------------------------------------

def attention_from_kv(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                      mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 softmax(q k^T / sqrt(d)) v for [B, H, Q, D] queries against [B, H, T, D]
    keys / values (core.py:800-820); masked-out positions get logit -1e9.
    Returns (output, weights)."""
    if min(query.ndim, keys.ndim, values.ndim) != 4 or max(query.ndim, keys.ndim, values.ndim) != 4:
        raise ValueError("query, keys, and values must be rank-4 tensors.")
    if keys.shape != values.shape:
        raise ValueError("keys and values must have the same shape.")
    if query.shape[:2] != keys.shape[:2] or query.shape[-1] != keys.shape[-1]:
        raise ValueError("query and KV batch/head/head_dim dimensions must match.")
    logits = torch.matmul(query.float(), keys.float().transpose(-2, -1)) / sqrt(query.size(-1))
    if mask is not None:
        keep = mask.to(device=logits.device, dtype=torch.bool)
        logits = logits.masked_fill(keep.logical_not(), -1.0e9)
    weights = logits.softmax(dim=-1)
    return torch.matmul(weights, values.float()), weights


def attention_report(query: torch.Tensor, original_keys: torch.Tensor, original_values: torch.Tensor,
                     quantized_layer: QuantizedKvLayer, mask: torch.Tensor | None = None) -> dict[str, float]:
    """How much the compression moves attention (core.py:823-845): output MSE,
    cosine and largest absolute change, and KL(original || compressed) of the
    weights (clamped at 1e-9), averaged over queries."""
    keys_q, values_q = quantized_layer.dequantize()
    dev = keys_q.device
    q = query.to(dev)
    out_ref, w_ref = attention_from_kv(q, original_keys.to(dev), original_values.to(dev), mask)
    out_q, w_q = attention_from_kv(q, keys_q, values_q, mask)
    p_ref, p_q = w_ref.clamp_min(1.0e-9), w_q.clamp_min(1.0e-9)
    kl = (p_ref * (p_ref.log() - p_q.log())).sum(dim=-1).mean()
    change = out_q - out_ref
    return {
        "attention_output_mse": float(F.mse_loss(out_q, out_ref).cpu()),
        "attention_output_cosine": _flat_cosine(out_q, out_ref),
        "attention_output_max_abs": float(change.abs().max().cpu()),
        "attention_weight_kl": float(kl.cpu()),
    }


def attention_from_quantized(query: torch.Tensor, quantized_layer: QuantizedKvLayer) -> torch.Tensor:
    """fp32 softmax(q k^T / sqrt(d)) v of [B, H, Q, D] queries (Q <= 16) over a
    compressed layer, read from its packed codes: the output of
    ``attention_from_kv(query, *quantized_layer.dequantize())[0]`` (core.py:800-820)
    without writing the dequantized keys and values.  The rows attended over are
    bit-identical to the dequantized cache's; the fp32 sums run in another order.
    Layers the attention kernels do not cover (passthrough layers, keys grouped
    along channels, head dims other than 64 / 128) are dequantized first."""
    if query.ndim != 4:
        raise ValueError("query, keys, and values must be rank-4 tensors.")
    B, H, T, D = quantized_layer.original_shape
    if tuple(query.shape[:2]) != (B, H) or query.shape[-1] != D:
        raise ValueError("query and KV batch/head/head_dim dimensions must match.")
    Q = query.shape[2]
    if quantized_layer.passthrough_keys is not None or Q > 16:
        keys, values = quantized_layer.dequantize()
        return attention_from_kv(query.to(keys.device), keys, values)[0]
    plan, _, _, dev = _run_plan([quantized_layer])
    lib = L.lib()
    ws_bytes = int(lib.gkv_attention_workspace_bytes(ctypes.byref(plan), B * H, Q))
    if ws_bytes == 0:
        keys, values = quantized_layer.dequantize()
        return attention_from_kv(query.to(keys.device), keys, values)[0]
    q = query.to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty((B, H, Q, D), dtype=torch.float32, device=dev)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        L.check(lib.gkv_attention(ctypes.byref(plan), B * H, q.data_ptr(), Q, out.data_ptr(), ws.data_ptr(),
                                  ws_bytes, L.stream_handle(dev)))
    return out


def _flat_cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    return float(F.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0).cpu())
