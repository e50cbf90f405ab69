"""CUDA path against the reference's own outputs (golden digests recorded from
the reference package on CPU) and against the numpy oracle.

Bar: index lists, packed codes, scale bit patterns, zero points, retained
rows and dequantized K/V are all compared byte-for-byte (sha256 of the
storage bits); on a mismatch the element-level difference is reported from
the stored arrays / the oracle.  The scores_ties case puts equal scores
across both selection boundaries, where the choice follows torch's CPU topk.
"""
import numpy as np
import pytest
import torch

from graphkv_b200 import QuantizedKvCache
from graphkv_b200 import _lib as L
from oracle import graphkv_oracle as orc
from tests.golden.cases import CASES, CASE_BY_NAME, bits_of, case_layers, case_scores, tensor_digest
from tests.helpers import config_for, layer_arrays
from tests.oracle_bridge import compare_arrays, load_golden, oracle_arrays, oracle_layers, reference_threads, scores_np

pytestmark = pytest.mark.gpu

SMALL = [c for c in CASES if not c.workload]
FULL = [c for c in CASES if c.workload and c.name != "w_qwen7b_8x131k_l0"]


def _to_cuda(scores):
    if scores is None:
        return None
    if isinstance(scores, list):
        return [s.cuda() for s in scores]
    return scores.cuda()


def _run(case, layers, scores, rec):
    pairs = [(k.cuda(), v.cuda()) for k, v in layers]
    with reference_threads(rec):  # the averaging of multi-dimensional scores follows the recorded thread count
        cache = QuantizedKvCache.from_past_key_values(pairs, config_for(case), _to_cuda(scores))
    deq = cache.dequantize()
    torch.cuda.synchronize()
    assert L.device_error() == 0
    return cache, deq


def _check_against_golden(case, cache, deq, rec, arrays):
    problems = []
    for li, layer in enumerate(cache.layers):
        problems += compare_arrays(case.name, layer_arrays(layer), rec["layers"][li], arrays, li)
        for n, d in zip("kv", deq[li]):
            if tensor_digest(bits_of(d)) != rec["layers"][li]["dequant"][n]:
                problems.append(f"l{li}: dequantized {n} differs from the reference")
        assert layer.stats() == rec["layers"][li]["layer_stats"]
    assert cache.stats() == rec["stats"]
    return problems


@pytest.mark.parametrize("case", SMALL, ids=lambda c: c.name)
def test_small_cases_match_reference(case):
    rec, arrays = load_golden(case.name)
    layers = case_layers(case)
    cache, deq = _run(case, layers, case_scores(case), rec)
    problems = _check_against_golden(case, cache, deq, rec, arrays)
    if problems:  # locate the first differing element against the oracle
        with reference_threads(rec):
            qls = oracle_layers(case, layers, scores_np(case_scores(case)))
        for li, ql in enumerate(qls):
            mine, ref = layer_arrays(cache.layers[li]), oracle_arrays(ql)
            for name in sorted(ref):
                if name in mine and not np.array_equal(mine[name].reshape(-1), ref[name].reshape(-1)):
                    bad = np.nonzero(mine[name].reshape(-1) != ref[name].reshape(-1))[0]
                    problems.append(f"vs oracle l{li} {name}: {bad.size} differ, first {bad[:4].tolist()}")
    assert not problems, problems


@pytest.mark.parametrize("case", FULL, ids=lambda c: c.name)
def test_full_workloads_match_reference(case):
    """Whole caches of the benchmark workloads (up to 28 x [1, 4, 32768, 128])."""
    rec, _ = load_golden(case.name)
    layers = case_layers(case)
    for li, (k, v) in enumerate(layers):
        assert tensor_digest(bits_of(k)) == rec["layers"][li]["inputs"]["k"], "input generation drifted"
    cache, deq = _run(case, layers, case_scores(case), rec)
    problems = _check_against_golden(case, cache, deq, rec, {})
    assert not problems, problems[:10]


@pytest.mark.slow
def test_batch8_131k_layer_matches_reference():
    """One layer of the 8 x 131072-token cache ([8, 4, 131072, 128] bf16)."""
    case = CASE_BY_NAME["w_qwen7b_8x131k_l0"]
    rec, _ = load_golden(case.name)
    layers = case_layers(case)
    cache, deq = _run(case, layers, case_scores(case), rec)
    problems = _check_against_golden(case, cache, deq, rec, {})
    assert not problems, problems[:10]
