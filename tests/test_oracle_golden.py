"""The numpy oracle against the reference's recorded outputs (CPU only)."""
import numpy as np
import pytest
import torch

from oracle import graphkv_oracle as orc
from tests.golden.cases import CASES, case_layers, case_scores, tensor_digest
from tests.oracle_bridge import compare_arrays, load_golden, oracle_arrays, oracle_layers, reference_threads, scores_np

SMALL = [c for c in CASES if not c.workload]


@pytest.mark.parametrize("case", SMALL, ids=lambda c: c.name)
def test_oracle_matches_reference(case):
    rec, arrays = load_golden(case.name)
    layers = case_layers(case)
    for li, (k, v) in enumerate(layers):
        from tests.golden.cases import bits_of
        assert tensor_digest(bits_of(k)) == rec["layers"][li]["inputs"]["k"], "input generation drifted"
    with reference_threads(rec):
        qls = oracle_layers(case, layers, scores_np(case_scores(case)))
    problems = []
    for li, ql in enumerate(qls):
        problems += compare_arrays(case.name, oracle_arrays(ql), rec["layers"][li], arrays, li)
        dk, dv = orc.dequantize_layer(ql)
        for n, d in (("k", dk), ("v", dv)):
            if tensor_digest(orc.storage_bits(d, ql.dtype)) != rec["layers"][li]["dequant"][n]:
                problems.append(f"l{li}: dequantized {n} differs")
        assert orc.layer_stats(ql) == rec["layers"][li]["layer_stats"]
    assert orc.cache_stats(qls) == rec["stats"]
    assert not problems, problems


def test_ties_case_has_boundary_ties():
    """The scores_ties golden exercises the tie rule: the k-th score also occurs
    outside the selected set, so torch's CPU topk order decides."""
    rec, _ = load_golden("scores_ties")
    assert rec["ties"]["protect"] is True


def test_pack_lowbit_known_answer():
    """Little-end-first packing: int4 symmetric [1, 2, 3, 0, -8, 7] -> 0xA9, 0x8B, 0xF0."""
    packed = orc.pack_lowbit(np.array([1, 2, 3, 0, -8, 7], np.int8), 4, -8)
    assert packed.tolist() == [0xA9, 0x8B, 0xF0]
    assert orc.unpack_lowbit(packed, 4, (6,), -8).tolist() == [1, 2, 3, 0, -8, 7]


def test_round_half_even_and_hadamard_division():
    x = np.array([0.5, 1.5, 2.5, -0.5, -1.5], np.float32)
    assert np.rint(x).tolist() == torch.round(torch.from_numpy(x)).tolist()
    y = np.random.default_rng(0).standard_normal((64, 128)).astype(np.float32)
    t = torch.from_numpy(y)
    ref = t
    h = 1
    while h < 128:  # the reference's butterflies, in torch
        ref = ref.reshape(64, 128 // (2 * h), 2, h)
        l, r = ref.unbind(dim=-2)
        ref = torch.stack((l + r, l - r), dim=-2).reshape(64, 128)
        h *= 2
    ref = (ref / np.sqrt(128)).numpy()
    assert np.array_equal(orc.hadamard_last_dim(y, "f32"), ref)
