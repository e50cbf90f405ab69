"""Averaging of multi-dimensional importance scores (core.py:1019-1031).

The reference averages [..., T] scores with reshape(-1, T).mean(0) and [T, ...]
scores with reshape(T, -1).mean(1).  On the CPU the last bit of each mean
depends on torch's summation order, and with it the tokens kept at a selection
boundary.  These CPU tests pin the oracle's restatement of that order against
torch itself (every thread count up to this host's), against the recorded
reference outputs, and check that the library's host-side block rule agrees
with the oracle's.  The GPU kernel is compared with the oracle in
test_gpu_score_mean.py.
"""
import os

import numpy as np
import pytest
import torch

from graphkv_b200.core import _sum_last_block
from oracle import graphkv_oracle as orc
from tests.golden.cases import CASE_BY_NAME, bits_of, case_layers, case_scores, tensor_digest
from tests.oracle_bridge import load_golden, policy_for, reference_threads, scores_np

SHAPES = [(2, 8192), (8, 4096), (8, 32768), (17, 5000), (64, 1024), (3, 100), (5, 7), (40, 33000),
          (100, 999), (512, 70), (1000, 33), (4096, 9), (8, 8197), (33, 8199)]
ADV = ["scores_rows64_adv", "scores_rows8_tail5", "scores_rows3d_adv", "scores_tx27_adv", "scores_tx5_adv",
       "scores_batch", "scores_heads"]


@pytest.mark.parametrize("threads", sorted({1, 2, 3, min(8, os.cpu_count() or 1), os.cpu_count() or 1}))
def test_restated_sum_order_equals_torch(threads):
    rng = np.random.default_rng(threads)
    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        for R, C in SHAPES:
            x = (rng.standard_normal((R, C)) * np.exp(3.0 * rng.standard_normal((R, C)))).astype(np.float32)
            for axis, xx in ((0, x), (1, np.ascontiguousarray(x.T))):
                ref = torch.from_numpy(xx).mean(axis).numpy()
                mine = (orc.torch_cpu_sum(xx, axis, threads) / np.float32(xx.shape[axis])).astype(np.float32)
                assert np.array_equal(ref.view(np.uint32), mine.view(np.uint32)), (threads, axis, xx.shape)
    finally:
        torch.set_num_threads(old)


def test_host_block_rule_matches_oracle():
    for threads in (1, 2, 3, 5, 8, 13, 24, 64, 96, 192):
        for R, C in SHAPES + [(8, 131072), (64, 131072), (1, 1048576), (3, 32768 * 3 + 17)]:
            assert _sum_last_block(R, C, threads) == orc.sum_last_block(R, C, threads), (threads, R, C)


@pytest.mark.parametrize("name", ADV)
def test_oracle_mean_equals_recorded_reference_mean(name):
    rec, arrays = load_golden(name)
    case = CASE_BY_NAME[name]
    T = case.shape[2]
    with reference_threads(rec):
        mine = orc.normalize_token_scores(T, scores_np(case_scores(case)))
    assert tensor_digest(mine.view(np.uint32)) == rec["score_mean"]


@pytest.mark.parametrize("name", ["scores_rows64_adv", "scores_rows3d_adv", "scores_tx27_adv", "scores_tx5_adv"])
def test_adversarial_cases_depend_on_the_summation_order(name):
    """With any other fp32 order (numpy's) the kept tokens differ from the
    reference's: the golden really pins the order."""
    rec, _ = load_golden(name)
    case = CASE_BY_NAME[name]
    T = case.shape[2]
    s = scores_np(case_scores(case))
    other = s.reshape(-1, T).mean(axis=0, dtype=np.float32) if case.scores != "tx_adv" else \
        s.reshape(T, -1).mean(axis=1, dtype=np.float32)
    with reference_threads(rec):
        exact = orc.normalize_token_scores(T, s)
    assert not np.array_equal(exact, other)
    p = policy_for(case)
    k, _ = case_layers(case)[0]
    ret_a, _, cold_a = orc.select_tiers(T, p, exact)
    ret_b, _, cold_b = orc.select_tiers(T, p, other)
    assert not (np.array_equal(ret_a, ret_b) and np.array_equal(cold_a, cold_b))
    assert tensor_digest(bits_of(torch.from_numpy(exact))) == rec["score_mean"]
