"""CPU oracle for the GraphKV cache-compression path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference package
``graphkv`` (``src/graphkv/core.py``) for the path ``quantize_hf_cache`` ->
``QuantizedKvCache`` -> ``dequantize`` / ``to_hf_dynamic_cache``.  It is the
checker that the CUDA path is compared against; it is never the thing that is
shipped or measured.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import it.

Parity pin: the restatement is checked against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference on CPU
and records its outputs) and against the eight byte totals the reference
publishes in ``README.md:25-30,125,128,131,134``.

Tensor representation.  numpy has no bfloat16, so every K/V tensor is held as a
float32 array whose values are exactly representable in its logical dtype
(``"bf16"``, ``"f16"`` or ``"f32"``); ``round_to`` performs the torch ``.to()``
cast (round-to-nearest-even) and returns float32 again.  All arithmetic is
float32 with IEEE round-to-nearest, matching torch's CPU kernels.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

F32 = np.float32
EPS = F32(1.0e-8)  # torch compares/clamps against the fp32 rounding of 1e-8 (core.py:869-871, 884)

DTYPE_SIZE = {"f32": 4, "f16": 2, "bf16": 2}


# ---------------------------------------------------------------------------
# dtype helpers
# ---------------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest, ties to even) and return the bit patterns."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32)
    rounded = ((b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded[nan] = ((b[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return rounded


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """torch ``Tensor.to(dtype)`` for a float32 tensor, returned as float32 values."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x)).reshape(x.shape)
    raise ValueError(dtype)


def storage_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """Bit patterns of ``x`` stored in ``dtype`` (for byte-exact comparisons)."""
    if dtype == "f32":
        return np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    if dtype == "f16":
        return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)
    return f32_to_bf16_bits(x)


# ---------------------------------------------------------------------------
# policy (mirrors KvQuantConfig, core.py:17-58, and the profiles, profiles.py:12-150)
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class Policy:
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
    scale_dtype: str = "f16"
    skip_if_not_smaller: bool = True


POLICIES = {
    # profiles.py:12-33
    "graphkv": Policy(bits=4, group_size=64, residual_length=256, sink_length=128, quantizer="affine",
                      long_context_threshold=8192, long_context_quantizer="symmetric",
                      semantic_protection_ratio=0.01, semantic_protection_min_context=8192,
                      semantic_residual_length=128, semantic_residual_min_context=8192,
                      low_priority_ratio=0.25, long_low_priority_ratio=0.35,
                      long_low_priority_min_context=32768, low_priority_min_context=8192,
                      low_priority_value_bits=2, low_priority_value_rotation="hadamard",
                      low_priority_value_rotation_min_context=32768),
    # profiles.py:74-86
    "graphkv-int2-max": Policy(bits=2, group_size=128, residual_length=0, quantizer="affine"),
    # profiles.py:87-99
    "graphkv-int4-balanced": Policy(bits=4, group_size=64, residual_length=0, quantizer="symmetric"),
    # profiles.py:100-115
    "graphkv-int4-safe": Policy(bits=4, group_size=64, residual_length=96, sink_length=32, quantizer="symmetric",
                                outlier_protection_ratio=0.02, min_outlier_tokens=1),
    # profiles.py:36-48
    "graphkv-qwen7-nf4": Policy(bits=4, group_size=32, residual_length=512, sink_length=128, quantizer="affine",
                                long_context_threshold=8192, long_context_quantizer="symmetric",
                                semantic_protection_ratio=0.02, semantic_protection_min_context=8192),
}


def effective_quantizer(p: Policy, T: int) -> str:
    """core.py:913-920."""
    if p.long_context_threshold is not None and p.long_context_quantizer is not None and T >= p.long_context_threshold:
        return p.long_context_quantizer
    return p.quantizer


def effective_low_priority_ratio(p: Policy, T: int) -> float:
    """core.py:923-929."""
    if p.long_low_priority_ratio is not None and T >= p.long_low_priority_min_context:
        return p.long_low_priority_ratio
    return p.low_priority_ratio


def effective_cold_value_rotation(p: Policy, T: int) -> str:
    """core.py:932-942 (fallback = the base rotation)."""
    if p.low_priority_value_rotation is not None and T >= p.low_priority_value_rotation_min_context:
        return p.low_priority_value_rotation
    return p.rotation


# ---------------------------------------------------------------------------
# selection (core.py:595-644, 685-719, 1019-1054)
# ---------------------------------------------------------------------------

def order_keys(scores: np.ndarray) -> np.ndarray:
    """Monotone uint32 keys for float32 scores: NaN is the largest value (torch.topk
    treats NaN as larger than any number) and -0.0 equals +0.0."""
    s = np.ascontiguousarray(scores, dtype=np.float32).copy()
    s[np.isnan(s)] = np.float32(np.nan)
    s[s == 0] = np.float32(0.0)
    b = s.view(np.uint32)
    neg = (b >> np.uint32(31)).astype(bool)
    return np.where(neg, ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def topk_indices(scores: np.ndarray, k: int, largest: bool) -> np.ndarray:
    """Positions of the k largest (or smallest) scores, as torch.topk on CPU
    chooses them (core.py:1047, 707).

    Without a tie at the k-th score the set is unique.  With one, torch's CPU
    topk (ATen ``TopKImpl.h``, ``topk_impl_loop``) decides by the order in which
    libstdc++ visits the (value, position) queue: ``std::partial_sort`` when
    ``k * 64 <= n``, else ``std::nth_element``; ``libstdc_select`` restates both."""
    keys = order_keys(scores)
    order = np.argsort(~keys if largest else keys, kind="stable")
    n = keys.size
    if k <= 0:
        return order[:0]
    if k >= n or keys[order[k - 1]] != keys[order[k]]:
        return order[:k]
    return np.asarray(libstdc_select(keys.tolist(), k, largest), dtype=np.int64)


# -- libstdc++ selection algorithms (GCC bits/stl_heap.h, bits/stl_algo.h) ---
# The comparator of ATen's topk is "x > y" (largest) or "x < y" (smallest) on
# the values, NaN ranked above every number; the order keys encode exactly that.

def _adjust_heap(q, first, hole, length, item, kv, less):
    """std::__adjust_heap then std::__push_heap: sift the hole at ``hole`` down
    to a leaf along the larger child (right child on ties), then push ``item`` up."""
    top = hole
    child = hole
    while child < (length - 1) // 2:
        child = 2 * (child + 1)
        if less(kv[q[first + child]], kv[q[first + child - 1]]):
            child -= 1
        q[first + hole] = q[first + child]
        hole = child
    if (length & 1) == 0 and child == (length - 2) // 2:
        child = 2 * (child + 1)
        q[first + hole] = q[first + child - 1]
        hole = child - 1
    parent = (hole - 1) // 2
    while hole > top and less(kv[q[first + parent]], kv[item]):
        q[first + hole] = q[first + parent]
        hole = parent
        parent = (hole - 1) // 2
    q[first + hole] = item


def _heap_select(q, first, middle, last, kv, less):
    """std::__heap_select: heapify [first, middle), then every later element that
    compares before the heap top replaces it (std::__pop_heap)."""
    length = middle - first
    if length >= 2:
        parent = (length - 2) // 2
        while True:
            _adjust_heap(q, first, parent, length, q[first + parent], kv, less)
            if parent == 0:
                break
            parent -= 1
    for i in range(middle, last):
        if less(kv[q[i]], kv[q[first]]):
            item = q[i]
            q[i] = q[first]
            _adjust_heap(q, first, 0, length, item, kv, less)


def _introselect(q, first, nth, last, kv, less):
    """std::__introselect with depth limit 2*floor(log2(n)): median-of-three
    pivot (first+1, middle, last-1) moved to ``first``, unguarded Hoare
    partition, recurse into the side holding ``nth``; heap select when the depth
    runs out; insertion sort of the final <= 3 elements."""
    depth = 2 * ((last - first).bit_length() - 1)
    while last - first > 3:
        if depth == 0:
            _heap_select(q, first, nth + 1, last, kv, less)
            q[first], q[nth] = q[nth], q[first]
            return
        depth -= 1
        a, b, c = first + 1, first + (last - first) // 2, last - 1
        ka, kb, kc = kv[q[a]], kv[q[b]], kv[q[c]]
        if less(ka, kb):
            m = b if less(kb, kc) else (c if less(ka, kc) else a)
        elif less(ka, kc):
            m = a
        elif less(kb, kc):
            m = c
        else:
            m = b
        q[first], q[m] = q[m], q[first]
        pivot = kv[q[first]]
        lo, hi = first + 1, last
        while True:
            while less(kv[q[lo]], pivot):
                lo += 1
            hi -= 1
            while less(pivot, kv[q[hi]]):
                hi -= 1
            if not lo < hi:
                break
            q[lo], q[hi] = q[hi], q[lo]
            lo += 1
        if lo <= nth:
            first = lo
        else:
            last = lo
    for i in range(first + 1, last):
        item = q[i]
        if less(kv[item], kv[q[first]]):
            q[first + 1:i + 1] = q[first:i]
            q[first] = item
        else:
            j = i
            while less(kv[item], kv[q[j - 1]]):
                q[j] = q[j - 1]
                j -= 1
            q[j] = item


def libstdc_select(keys: list, k: int, largest: bool) -> list:
    """Positions that end in the first k slots of torch's CPU topk queue."""
    n = len(keys)
    q = list(range(n))
    less = (lambda x, y: x > y) if largest else (lambda x, y: x < y)
    if k * 64 <= n:
        _heap_select(q, 0, k, n, keys, less)
    else:
        _introselect(q, 0, k - 1, n, keys, less)
    return sorted(q[:k])


def boundary_tie(scores: np.ndarray, k: int, largest: bool) -> bool:
    """True when the k-th selected score also occurs outside the selected set."""
    if k <= 0 or k >= scores.size:
        return False
    keys = order_keys(scores)
    order = np.argsort(~keys if largest else keys, kind="stable")
    return bool(keys[order[k - 1]] == keys[order[k]])


# ---------------------------------------------------------------------------
# torch's CPU fp32 sum, restated in its summation order.  The reference averages
# [..., T] / [T, ...] scores with Tensor.mean (core.py:1027-1030), which on the CPU
# is sum (ATen's cascade_sum, native/cpu/SumKernel.cpp) followed by one division
# by the element count.  The order of the fp32 additions is:
#  * cascade (multi_row_sum): rows are added one by one into level 0; after every
#    2^p rows (p = max(4, ceil_log2(n) // 4)) level j-1 is folded into level j
#    while the row count is a multiple of 2^(p*j); leftover rows go into level 0;
#    finally level 0 += level 1, += level 2, += level 3;
#  * row_sum: four interleaved cascades over rows 4i+k, leftover rows added to
#    partial 0, then partial 0 += partial 1, += 2, += 3;
#  * outer reduction ([R, T] over R): columns are split into per-thread blocks
#    (at::parallel_for over columns, block ends rounded down to 32 columns unless
#    at the end); inside a block, whole groups of 32 columns take the cascade and
#    the rest of the block takes row_sum (a block narrower than 8 columns: whole
#    groups of 4 columns cascade);
#  * inner reduction ([T, X] over X): 8-lane vectors (the sum kernel is the AVX2
#    one on every x86 host), lane l is a row_sum over elements 8v + l, the
#    leftover X % 8 elements are added into a scalar starting at 0, followed by
#    lanes 0..7; X < 8: one scalar row_sum;
#  * the output is pre-filled with 0 and receives 0 + sum.
# ---------------------------------------------------------------------------
SUM_LANES = 8
SUM_GRAIN = 32768      # at::internal::GRAIN_SIZE
SUM_THREADS = 1        # at::get_num_threads() of the process that ran the reference (set by the tests)


def _ceil_log2(x: int) -> int:
    return 1 if x <= 2 else int(x - 1).bit_length()


def _cascade(rows: list) -> np.ndarray:
    n = len(rows)
    p = max(4, _ceil_log2(n) // 4)
    step, mask = 1 << p, (1 << p) - 1
    acc = [np.zeros_like(rows[0]) for _ in range(4)]
    i = 0
    while i + step <= n:
        for _ in range(step):
            acc[0] = (acc[0] + rows[i]).astype(F32)
            i += 1
        for j in range(1, 4):
            acc[j] = (acc[j] + acc[j - 1]).astype(F32)
            acc[j - 1] = np.zeros_like(acc[j - 1])
            if i & (mask << (j * p)):
                break
    while i < n:
        acc[0] = (acc[0] + rows[i]).astype(F32)
        i += 1
    for j in range(1, 4):
        acc[0] = (acc[0] + acc[j]).astype(F32)
    return acc[0]


def _row_sum(rows: list) -> np.ndarray:
    n4 = len(rows) // 4
    parts = [_cascade(rows[k::4][:n4]) if n4 else np.zeros_like(rows[0]) for k in range(4)]
    for i in range(4 * n4, len(rows)):
        parts[0] = (parts[0] + rows[i]).astype(F32)
    for k in range(1, 4):
        parts[0] = (parts[0] + parts[k]).astype(F32)
    return parts[0]


def sum_last_block(rows: int, cols: int, threads: int) -> int:
    """First column of the last per-thread block of an outer reduction."""
    if rows * cols < SUM_GRAIN or threads <= 1 or cols <= 1:
        return 0
    nt = min(threads, cols)
    cs = -(-cols // nt)
    last = 0
    for tid in range(nt):
        b, e = tid * cs, min(cols, tid * cs + cs)
        if b >= cols:
            continue
        b -= b % 32
        if e != cols:
            e -= e % 32
        if b < e:
            last = b
    return last


def torch_cpu_sum(x: np.ndarray, axis: int, threads: int) -> np.ndarray:
    """Sum of a contiguous fp32 [R, C] array over `axis` in torch's CPU order."""
    x = np.ascontiguousarray(x, dtype=F32)
    if axis == 0:
        R, C = x.shape
        out = np.zeros(C, F32)
        blocks, b0 = [], 0
        last = sum_last_block(R, C, threads)
        for b in range(0, last, 32):  # blocks before the last one are whole 32-column groups
            blocks.append((b, b + 32))
        blocks.append((last, C))
        for b, e in blocks:
            n = e - b
            if n >= SUM_LANES:
                a_end = n // (4 * SUM_LANES) * (4 * SUM_LANES)
            else:
                a_end = n // 4 * 4
            rows = [x[r, b:e] for r in range(R)]
            res = np.empty(n, F32)
            if a_end:
                res[:a_end] = _cascade([r[:a_end] for r in rows])
            if n > a_end:
                res[a_end:] = _row_sum([r[a_end:] for r in rows])
            out[b:e] = (out[b:e] + res).astype(F32)
        return out
    T, X = x.shape
    cols = [x[:, c] for c in range(X)]
    if X >= SUM_LANES:
        nv = X // SUM_LANES
        fin = np.zeros(T, F32)
        for c in range(nv * SUM_LANES, X):
            fin = (fin + cols[c]).astype(F32)
        for lane in range(SUM_LANES):
            fin = (fin + _row_sum([cols[v * SUM_LANES + lane] for v in range(nv)])).astype(F32)
    else:
        fin = _row_sum(cols)
    return (np.zeros(T, F32) + fin).astype(F32)


def normalize_token_scores(T: int, scores: np.ndarray, threads: Optional[int] = None) -> np.ndarray:
    """core.py:1019-1031: scores as fp32 [T]; [..., T] and [T, ...] scores are
    averaged over the other dimension as torch's CPU mean does (sum in the order
    above, then one fp32 division by the count)."""
    s = np.asarray(scores, dtype=np.float32)
    th = SUM_THREADS if threads is None else threads
    if s.size == T:
        return s.reshape(T)
    if s.ndim >= 1 and s.shape[-1] == T:
        x = s.reshape(-1, T)
        return (torch_cpu_sum(x, 0, th) / F32(x.shape[0])).astype(F32)
    if s.ndim >= 1 and s.shape[0] == T:
        x = s.reshape(T, -1)
        return (torch_cpu_sum(x, 1, th) / F32(x.shape[1])).astype(F32)
    raise ValueError("importance_scores must have one score per token or a final token dimension.")


def keep_count(n: int, ratio: float, minimum: int) -> int:
    """core.py:1044 and 702-705."""
    return min(n, max(math.ceil(n * ratio), minimum))


def apply_score_retention(mask: np.ndarray, scores: np.ndarray, candidates: np.ndarray, ratio: float, minimum: int) -> None:
    """core.py:1034-1048."""
    cand = np.nonzero(candidates)[0]
    keep = keep_count(int(cand.size), ratio, minimum)
    if keep <= 0:
        return
    top = topk_indices(scores[cand], keep, largest=True)
    mask[cand[top]] = True


def retention_mask(T: int, p: Policy, scores: Optional[np.ndarray]) -> np.ndarray:
    """core.py:595-644."""
    mask = np.zeros(T, dtype=bool)
    sink = min(p.sink_length, T)
    if sink:
        mask[:sink] = True
    residual = p.residual_length
    if scores is not None and p.semantic_residual_length is not None and T >= p.semantic_residual_min_context:
        residual = p.semantic_residual_length
    residual = min(residual, T)
    if residual:
        mask[T - residual:] = True
    candidates = ~mask
    if scores is None or T < p.semantic_protection_min_context or not candidates.any():
        return mask
    apply_score_retention(mask, normalize_token_scores(T, scores), candidates,
                          p.semantic_protection_ratio, p.min_protected_tokens)
    return mask


def outlier_scores(K: np.ndarray, V: np.ndarray) -> np.ndarray:
    """core.py:1051-1054: mean of squares over (batch, heads, head_dim) per token."""
    k = np.square(K.astype(np.float32)).mean(axis=(0, 1, 3), dtype=np.float32)
    v = np.square(V.astype(np.float32)).mean(axis=(0, 1, 3), dtype=np.float32)
    return (k + v).astype(np.float32)


def select_tiers(T: int, p: Policy, scores: Optional[np.ndarray], K=None, V=None):
    """Index lists (int32, ascending) for retained / standard / cold tokens.
    core.py:668-719."""
    mask = retention_mask(T, p, scores)
    if p.outlier_protection_ratio > 0.0 or p.min_outlier_tokens > 0:
        apply_score_retention(mask, outlier_scores(K, V), ~mask, p.outlier_protection_ratio, p.min_outlier_tokens)
    compressed = ~mask
    cold = np.zeros(T, dtype=bool)
    ratio = effective_low_priority_ratio(p, T)
    if (scores is not None and T >= p.low_priority_min_context
            and (ratio > 0.0 or p.min_low_priority_tokens > 0)
            and (p.low_priority_bits is not None or p.low_priority_key_bits is not None
                 or p.low_priority_value_bits is not None)
            and compressed.any()):
        s = normalize_token_scores(T, scores)
        cand = np.nonzero(compressed)[0]
        keep = keep_count(int(cand.size), ratio, p.min_low_priority_tokens)
        if keep > 0:
            cold[cand[topk_indices(s[cand], keep, largest=False)]] = True
    standard = compressed & ~cold
    ar = np.arange(T)
    return ar[mask].astype(np.int32), ar[standard].astype(np.int32), ar[cold].astype(np.int32)


# ---------------------------------------------------------------------------
# Hadamard rotation, quantization, packing (core.py:848-910, 945-956, 979-1007)
# ---------------------------------------------------------------------------

def hadamard_last_dim(x: np.ndarray, out_dtype: str) -> np.ndarray:
    """core.py:945-956: Sylvester butterflies h = 1, 2, 4, ... in fp32, then an
    fp32 division by fp32(sqrt(D)), then the cast back to the input dtype."""
    D = x.shape[-1]
    if D < 1 or D & (D - 1):
        raise ValueError("hadamard rotation requires a power-of-two head dimension.")
    lead = x.shape[:-1]
    y = np.ascontiguousarray(x, dtype=np.float32)
    h = 1
    while h < D:
        y = y.reshape(*lead, D // (2 * h), 2, h)
        left, right = y[..., 0, :], y[..., 1, :]
        y = np.stack((left + right, left - right), axis=-2).reshape(*lead, D)
        h *= 2
    return round_to(y / F32(math.sqrt(D)), out_dtype)


@dataclass
class QTensor:
    """Mirror of QuantizedTensor (core.py:130-151)."""
    q: np.ndarray             # packed uint8 stream, or int8/uint8 codes when unpacked
    scales: np.ndarray        # float32 values of the stored scales, shape [..., ngroups, 1]
    scale_dtype: str
    zero_points: Optional[np.ndarray]
    original_shape: tuple
    axis: int
    group_size: int
    bits: int
    padded: int
    q_shape: tuple
    original_dtype: str
    packed: bool
    packed_offset: int
    rotation: str = "none"

    def memory_bytes(self) -> int:
        """core.py:150-151."""
        n = self.q.size * self.q.itemsize + self.scales.size * DTYPE_SIZE[self.scale_dtype]
        if self.zero_points is not None:
            n += self.zero_points.size
        return n

    def scale_bits(self) -> np.ndarray:
        return storage_bits(self.scales, self.scale_dtype)


def pack_lowbit(q: np.ndarray, bits: int, offset: int) -> np.ndarray:
    """core.py:979-990: flatten, subtract the offset, element i goes to bits i*bits of its byte."""
    vpb = 8 // bits
    enc = (q.astype(np.int16) - offset).astype(np.uint8).reshape(-1)
    pad = (-enc.size) % vpb
    if pad:
        enc = np.concatenate([enc, np.zeros(pad, np.uint8)])
    enc = enc.reshape(-1, vpb)
    out = np.zeros(enc.shape[0], dtype=np.uint8)
    for i in range(vpb):
        out |= (enc[:, i] << np.uint8(i * bits)).astype(np.uint8)
    return out


def unpack_lowbit(packed: np.ndarray, bits: int, q_shape: tuple, offset: int) -> np.ndarray:
    """core.py:993-1007."""
    vpb = 8 // bits
    mask = (1 << bits) - 1
    parts = [(packed >> np.uint8(i * bits)) & np.uint8(mask) for i in range(vpb)]
    enc = np.stack(parts, axis=1).reshape(-1)[: int(np.prod(q_shape))]
    q = enc.astype(np.int16) + offset
    return (q.astype(np.uint8) if offset == 0 else q.astype(np.int8)).reshape(q_shape)


def quantize_tensor(x: np.ndarray, dtype: str, bits: int, group_size: int, quantizer: str, axis: int,
                    rotation: str = "none", pack_int4: bool = True, scale_dtype: str = "f16") -> QTensor:
    """core.py:848-910."""
    if rotation == "hadamard":
        x = hadamard_last_dim(x, dtype)
    axis = axis % x.ndim
    moved = np.ascontiguousarray(np.moveaxis(x, axis, -1), dtype=np.float32)
    n = moved.shape[-1]
    gs = min(group_size, n)
    padded = (-n) % gs
    if padded:
        moved = np.concatenate([moved, np.zeros((*moved.shape[:-1], padded), np.float32)], axis=-1)
    q_shape = tuple(moved.shape)
    g = moved.reshape(*q_shape[:-1], q_shape[-1] // gs, gs)
    if quantizer == "affine":
        qmax = (1 << bits) - 1
        mins = g.min(axis=-1, keepdims=True)
        maxs = g.max(axis=-1, keepdims=True)
        ranges = (maxs - mins).astype(np.float32)
        degenerate = ranges < EPS
        fallback = np.maximum(np.abs(g).max(axis=-1, keepdims=True), EPS) / F32(qmax)
        scales = np.where(degenerate, fallback, np.maximum(ranges, EPS) / F32(qmax)).astype(np.float32)
        zpf = np.clip(np.rint(-mins / scales), 0, qmax)
        zp = np.where(degenerate, np.where(mins < 0, F32(qmax), F32(0)), zpf).astype(np.uint8)
        q = np.clip(np.rint(g / scales + zp.astype(np.float32)), 0, qmax).astype(np.uint8)
        offset = 0
    else:
        qmax = (1 << (bits - 1)) - 1
        qmin = -(1 << (bits - 1))
        scales = (np.maximum(np.abs(g).max(axis=-1, keepdims=True), EPS) / F32(qmax)).astype(np.float32)
        zp = None
        q = np.clip(np.rint(g / scales), qmin, qmax).astype(np.int8)
        offset = qmin
    q = q.reshape(q_shape)
    packed = bits in (2, 4) and pack_int4
    return QTensor(q=pack_lowbit(q, bits, offset) if packed else q,
                   scales=round_to(scales, scale_dtype), scale_dtype=scale_dtype,
                   zero_points=zp, original_shape=tuple(x.shape), axis=axis, group_size=gs, bits=bits,
                   padded=padded, q_shape=q_shape, original_dtype=dtype, packed=packed,
                   packed_offset=offset, rotation=rotation)


def dequantize_tensor(t: QTensor) -> np.ndarray:
    """core.py:153-173; returns float32 values of the original dtype."""
    q = unpack_lowbit(t.q, t.bits, t.q_shape, t.packed_offset) if t.packed else t.q.reshape(t.q_shape)
    gshape = (*t.q_shape[:-1], t.q_shape[-1] // t.group_size, t.group_size)
    g = q.reshape(gshape).astype(np.float32)
    if t.zero_points is not None:
        g = g - t.zero_points.astype(np.float32)
    g = g * t.scales.astype(np.float32)
    moved = g.reshape(t.q_shape)
    if t.padded:
        moved = moved[..., : t.original_shape[t.axis]]
    out = np.ascontiguousarray(np.moveaxis(moved, -1, t.axis))
    if t.rotation == "hadamard":
        out = hadamard_last_dim(out, "f32")
    return round_to(out, t.original_dtype)


# ---------------------------------------------------------------------------
# layer orchestration and accounting (core.py:176-263, 647-772, 959-976)
# ---------------------------------------------------------------------------

@dataclass
class QLayer:
    original_shape: tuple
    dtype: str
    idx_ret: np.ndarray
    idx_std: np.ndarray
    idx_cold: np.ndarray
    ret_k: np.ndarray
    ret_v: np.ndarray
    std_k: Optional[QTensor] = None
    std_v: Optional[QTensor] = None
    cold_k: Optional[QTensor] = None
    cold_v: Optional[QTensor] = None
    passthrough: Optional[tuple] = None
    tensors: dict = field(default_factory=dict)

    def memory_bytes(self) -> int:
        """core.py:194-215."""
        if self.passthrough is not None:
            return 2 * self.passthrough[0].size * DTYPE_SIZE[self.dtype]
        n = 0
        for t in (self.std_k, self.std_v, self.cold_k, self.cold_v):
            if t is not None:
                n += t.memory_bytes()
        n += 4 * (self.idx_ret.size + self.idx_std.size + self.idx_cold.size)
        n += (self.ret_k.size + self.ret_v.size) * DTYPE_SIZE[self.dtype]
        return n

    def original_memory_bytes(self) -> int:
        """core.py:217-226."""
        return 2 * int(np.prod(self.original_shape)) * DTYPE_SIZE[self.dtype]

    def counts(self):
        if self.passthrough is not None:
            return self.original_shape[2], 0, 0
        return int(self.idx_ret.size), int(self.idx_std.size), int(self.idx_cold.size)


def quantize_layer(K: np.ndarray, V: np.ndarray, dtype: str, p: Policy,
                   scores: Optional[np.ndarray] = None) -> QLayer:
    """core.py:647-772 for K/V of layout [B, H, T, D]."""
    if K.shape != V.shape:
        raise ValueError("keys and values must have the same shape.")
    if K.ndim != 4:
        raise ValueError("keys and values must use [batch, heads, tokens, head_dim] layout.")
    T = K.shape[2]
    quantizer = effective_quantizer(p, T)
    idx_ret, idx_std, idx_cold = select_tiers(T, p, scores, K, V)
    key_axis = 2 if p.key_group_axis == "token" else 3
    value_axis = 2 if p.value_group_axis == "token" else 3
    layer = QLayer(original_shape=tuple(K.shape), dtype=dtype, idx_ret=idx_ret, idx_std=idx_std,
                   idx_cold=idx_cold, ret_k=K[:, :, idx_ret, :], ret_v=V[:, :, idx_ret, :])
    common = dict(quantizer=quantizer, pack_int4=p.pack_int4, scale_dtype=p.scale_dtype, group_size=p.group_size)
    if idx_std.size:
        layer.std_k = quantize_tensor(K[:, :, idx_std, :], dtype, p.key_bits or p.bits, axis=key_axis,
                                      rotation=p.rotation, **common)
        layer.std_v = quantize_tensor(V[:, :, idx_std, :], dtype, p.value_bits or p.bits, axis=value_axis,
                                      rotation=p.rotation, **common)
    if idx_cold.size:
        low = p.low_priority_bits or p.bits
        layer.cold_k = quantize_tensor(K[:, :, idx_cold, :], dtype, p.low_priority_key_bits or low,
                                       axis=key_axis, rotation=p.rotation, **common)
        layer.cold_v = quantize_tensor(V[:, :, idx_cold, :], dtype, p.low_priority_value_bits or low,
                                       axis=value_axis, rotation=effective_cold_value_rotation(p, T), **common)
    if p.skip_if_not_smaller and layer.memory_bytes() >= layer.original_memory_bytes():
        e = np.zeros(0, np.int32)
        return QLayer(original_shape=tuple(K.shape), dtype=dtype, idx_ret=e, idx_std=e, idx_cold=e,
                      ret_k=K[:, :, :0, :], ret_v=V[:, :, :0, :], passthrough=(K, V))
    return layer


def dequantize_layer(layer: QLayer):
    """core.py:265-307: every output row is written from exactly one tier."""
    if layer.passthrough is not None:
        return layer.passthrough
    K = np.empty(layer.original_shape, np.float32)
    V = np.empty(layer.original_shape, np.float32)
    if layer.std_k is not None and layer.idx_std.size:
        K[:, :, layer.idx_std, :] = dequantize_tensor(layer.std_k)
        V[:, :, layer.idx_std, :] = dequantize_tensor(layer.std_v)
    if layer.cold_k is not None and layer.idx_cold.size:
        K[:, :, layer.idx_cold, :] = dequantize_tensor(layer.cold_k)
        V[:, :, layer.idx_cold, :] = dequantize_tensor(layer.cold_v)
    if layer.idx_ret.size:
        K[:, :, layer.idx_ret, :] = layer.ret_k
        V[:, :, layer.idx_ret, :] = layer.ret_v
    return K, V


def layer_stats(layer: QLayer) -> dict:
    """core.py:231-248."""
    orig, comp = layer.original_memory_bytes(), layer.memory_bytes()
    r, c, l = layer.counts()
    comp_tokens = c + l
    total = r + comp_tokens
    return {
        "original_bytes": float(orig),
        "compressed_bytes": float(comp),
        "compression_ratio": orig / max(comp, 1),
        "retained_tokens": float(r),
        "compressed_tokens": float(comp_tokens),
        "standard_compressed_tokens": float(c),
        "low_priority_tokens": float(l),
        "retained_fraction": r / max(total, 1),
        "compressed_fraction": comp_tokens / max(total, 1),
    }


def cache_stats(layers: list) -> dict:
    """core.py:392-413."""
    orig = sum(l.original_memory_bytes() for l in layers)
    comp = sum(l.memory_bytes() for l in layers)
    r = sum(l.counts()[0] for l in layers)
    c = sum(l.counts()[1] for l in layers)
    lp = sum(l.counts()[2] for l in layers)
    comp_tokens = c + lp
    total = r + comp_tokens
    ratios = [l.original_memory_bytes() / max(l.memory_bytes(), 1) for l in layers]
    return {
        "layers": float(len(layers)),
        "original_bytes": float(orig),
        "compressed_bytes": float(comp),
        "compression_ratio": orig / max(comp, 1),
        "retained_tokens": float(r),
        "compressed_tokens": float(comp_tokens),
        "standard_compressed_tokens": float(c),
        "low_priority_tokens": float(lp),
        "retained_fraction": r / max(total, 1),
        "compressed_fraction": comp_tokens / max(total, 1),
        "min_layer_compression_ratio": min(ratios, default=0.0),
        "max_layer_compression_ratio": max(ratios, default=0.0),
    }


def layer_tensors(layer: QLayer) -> dict:
    """Flat dictionary of every stored array of a layer, in storage form, for
    byte-exact comparison: packed codes, scale bit patterns, zero points,
    index lists and the retained rows' bit patterns."""
    out = {"idx_ret": layer.idx_ret, "idx_std": layer.idx_std, "idx_cold": layer.idx_cold,
           "ret_k": storage_bits(layer.ret_k, layer.dtype), "ret_v": storage_bits(layer.ret_v, layer.dtype)}
    for name in ("std_k", "std_v", "cold_k", "cold_v"):
        t = getattr(layer, name)
        if t is None:
            continue
        out[name + ".q"] = t.q
        out[name + ".scales"] = t.scale_bits()
        if t.zero_points is not None:
            out[name + ".zp"] = t.zero_points
    return out
