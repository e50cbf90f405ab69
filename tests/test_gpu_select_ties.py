"""Tier selection when equal scores straddle a selection boundary.

The reference selects with torch.topk on the CPU, whose choice among equal
scores follows the order libstdc++'s partial_sort (k * 64 <= n) or
nth_element visits the candidate queue.  The CUDA select kernel reproduces
that order; these tests call it through the C ABI (gkv_select_tiers) on
tie-heavy scores and compare the three index lists with the oracle's
restatement (integer outputs: exact equality).  Both regimes are reached for
the largest (protection) and the smallest (cold tier) selection, in the
shared-memory variant of the kernel (at most 40960 tokens per block of its
8-block cluster) and in the global-memory variant (longer sequences), with
ties inside one block's range and across the ranges of several blocks.
"""
import ctypes
from dataclasses import replace

import numpy as np
import pytest
import torch

from graphkv_b200 import _lib as L
from graphkv_b200.config import resolve_tiers
from graphkv_b200.profiles import get_profile
from oracle import graphkv_oracle as orc

pytestmark = pytest.mark.gpu


def _scores(T: int, kind: str, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind.startswith("levels"):
        return rng.integers(0, int(kind[6:]), T).astype(np.float32)
    if kind == "chunks":  # graph-memory shape: runs of one score, 0 between them
        s = np.zeros(T, np.float32)
        for _ in range(24):
            a = int(rng.integers(0, T - 64))
            s[a:a + int(rng.integers(16, max(17, T // 16)))] = np.float32(rng.integers(1, 6) / 5)
        return s
    if kind == "specials":  # NaN ranks highest, -0.0 equals +0.0
        s = rng.integers(-2, 3, T).astype(np.float32)
        s[rng.integers(0, T, T // 50)] = np.nan
        s[s == 0] = np.float32(-0.0)
        s[rng.integers(0, T, T // 7)] = np.float32(0.0)
        return s
    if kind == "sorted":
        return np.sort(rng.integers(0, 9, T).astype(np.float32))
    if kind == "lognormal":  # continuous: no tie at either boundary
        return np.exp(2.0 * rng.standard_normal(T)).astype(np.float32)
    raise ValueError(kind)


def _gpu_select(scores: np.ndarray, tiers) -> tuple:
    lib = L.lib()
    T = tiers.seq_len
    s = torch.from_numpy(scores).cuda()
    idx = torch.full((T,), -1, dtype=torch.int32, device="cuda")
    r, st, c = torch.split(idx, [tiers.n_retained, tiers.n_standard, tiers.n_cold])
    ws = torch.empty(int(lib.gkv_select_workspace_bytes(T)), dtype=torch.uint8, device="cuda")
    pol = tiers.policy()
    L.check(lib.gkv_select_tiers(s.data_ptr(), None, ctypes.byref(pol), r.data_ptr(), st.data_ptr(), c.data_ptr(),
                                 ws.data_ptr(), ws.numel(), L.stream_handle(s.device)))
    torch.cuda.synchronize()
    assert L.device_error() == 0
    return r.cpu().numpy(), st.cpu().numpy(), c.cpu().numpy()


CASES = [
    # T, profile, overrides, scores
    (9000, "graphkv", {}, "levels3"),
    (20000, "graphkv", {}, "levels50"),
    (40960, "graphkv", {}, "chunks"),
    (32768, "graphkv", {}, "levels2"),
    (50000, "graphkv", {}, "levels7"),
    (131072, "graphkv", {}, "levels1000"),
    (131072, "graphkv", {}, "chunks"),
    (32768, "graphkv", {}, "lognormal"),
    (393216, "graphkv", {}, "lognormal"),
    (393216, "graphkv", {}, "levels5000"),
    (100, "graphkv", {"sink_length": 8, "residual_length": 8, "semantic_protection_min_context": 64,
                      "low_priority_min_context": 64}, "levels3"),
    (12000, "graphkv-qwen7-nf4", {}, "levels4"),
    (16384, "graphkv", {}, "specials"),
    (16384, "graphkv", {}, "sorted"),
    # protection in the nth_element regime, cold tier in the partial_sort regime
    (10000, "graphkv", {"semantic_protection_ratio": 0.3, "low_priority_ratio": 0.01}, "levels5"),
    (60000, "graphkv", {"semantic_protection_ratio": 0.5, "long_low_priority_ratio": 0.005}, "levels20"),
    (8192, "graphkv", {"min_protected_tokens": 5000}, "levels3"),
    # shared-memory variant whose heap (4497 nodes) does not fit beside the block's
    # tokens: the heap select keeps its nodes in the workspace
    (300000, "graphkv", {"semantic_protection_ratio": 0.015}, "levels200"),
]


def _adversarial(n: int, k: int, largest: bool) -> np.ndarray:
    """Scores that drive introselect into its depth limit (heap-select
    fallback), with equal scores across the k-th position: M. D. McIlroy's
    adversary ("A killer adversary for quicksort", 1999) run against the
    oracle's restatement, then the scores around rank k merged into one."""
    gas = n
    val = [gas] * n
    state = {"solid": 0, "cand": -1}

    def freeze(x):
        val[x] = state["solid"]
        state["solid"] += 1

    def less(x, y):
        if val[x] == gas and val[y] == gas:
            freeze(x if x == state["cand"] else y)
        if val[x] == gas:
            state["cand"] = x
        elif val[y] == gas:
            state["cand"] = y
        return val[x] > val[y] if largest else val[x] < val[y]

    orc._introselect(list(range(n)), 0, k - 1, n, list(range(n)), less)
    for i in range(n):
        if val[i] == gas:
            freeze(i)
    v = np.array(val, np.float32)
    order = np.argsort(-v if largest else v, kind="stable")
    v[order[k - 4:k + 4]] = v[order[k - 1]]
    return v


def _policy(n: int, k: int, largest: bool) -> L.SelectPolicy:
    if largest:
        return L.SelectPolicy(n, 0, 0, k, 0, 0, k, n - k, 0, 0)
    return L.SelectPolicy(n, 0, 0, 0, 0, k, 0, n - k, k, 0)


class _Tiers:  # the host-side policy of a raw selection
    def __init__(self, pol):
        self.pol = pol
        self.seq_len, self.n_retained, self.n_standard, self.n_cold = pol.seq_len, pol.n_retained, pol.n_standard, \
            pol.n_cold

    def policy(self):
        return self.pol


@pytest.mark.parametrize("n,k,largest", [(2000, 1000, False), (2000, 700, True), (5000, 2000, False),
                                         (60000, 30000, True)])
def test_introselect_depth_limit_fallback(n, k, largest):
    scores = _adversarial(n, k, largest)
    got = _gpu_select(scores, _Tiers(_policy(n, k, largest)))
    want = np.sort(orc.topk_indices(scores, k, largest)).astype(np.int32)
    assert np.array_equal(got[0] if largest else got[2], want)


@pytest.mark.parametrize("T,profile,over,kind", CASES,
                         ids=[f"{c[0]}-{c[1]}-{c[3]}{'-' + '-'.join(c[2]) if c[2] else ''}" for c in CASES])
def test_tie_selection_matches_cpu_topk_order(T, profile, over, kind):
    cfg = replace(get_profile(profile).config, **over)
    pol = replace(orc.POLICIES[profile], **over)
    scores = _scores(T, kind, seed=T + len(kind))
    ref = orc.select_tiers(T, pol, scores)
    tiers = resolve_tiers(cfg, T, True)
    got = _gpu_select(scores, tiers)
    for name, a, b in zip(("retained", "standard", "cold"), got, ref):
        assert np.array_equal(a, b), f"{name}: {np.setdiff1d(a, b)[:8]} vs {np.setdiff1d(b, a)[:8]}"
