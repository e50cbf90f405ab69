"""Graph Mneme scoring (``quantize_hf_cache(graph_memory=...)``) against the
reference's recorded outputs (``tests/golden/graph_mneme.json``).

CPU: parameter names/shapes (checkpoint compatibility), fact banks, raw chunk
scores and token scores are compared bit-for-bit; the oracle's selection over
those token scores must equal the reference's index lists (graph scores tie
across whole chunks, so this exercises the torch.topk tie order).
GPU: the whole request path through the CUDA selection and quantizer.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from graphkv_b200 import graph_model as gm
from oracle import graphkv_oracle as orc
from tests.golden.graph_cases import GRAPH_CASES, build_model, build_request, cache_layers

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = json.load(open(os.path.join(HERE, "golden", "graph_mneme.json")))
RECORDS = {r["case"]: r for r in GOLDEN["cases"]}
CASE_IDS = [c.name for c in GRAPH_CASES]


def _digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _banks(model, req):
    q = gm.build_query_bank(req.query_anchor, req.query_relation, req.query_facts, model.cfg,
                            shuffle_seed=req.shuffle_seed)
    cands = [gm.build_candidate_bank(ch.anchor, ch.facts, model.cfg, shuffle_seed=ch.shuffle_seed)
             for ch in req.chunks]
    return q, cands


def _bank_record(bank):
    return {"src": bank.src.tolist(), "rel": bank.rel.tolist(), "dst": bank.dst.tolist(),
            "entity_map": [list(x) for x in sorted(bank.entity_map.items())],
            "relation_map": [list(x) for x in sorted(bank.relation_map.items())]}


@pytest.mark.parametrize("case", GRAPH_CASES, ids=CASE_IDS)
def test_parameters_match_reference_checkpoint_layout(case):
    model = build_model(gm, case)
    mine = [[k, list(v.shape)] for k, v in sorted(model.state_dict().items())]
    assert mine == RECORDS[case.name]["params"]


@pytest.mark.parametrize("case", GRAPH_CASES, ids=CASE_IDS)
def test_fact_banks_match_reference(case):
    rec = RECORDS[case.name]
    model, req = build_model(gm, case), build_request(gm, case)
    q, cands = _banks(model, req)
    assert _bank_record(q.facts) == rec["query"]
    assert q.query_relation == rec["query_relation"]
    assert [_bank_record(b) for b in cands] == rec["candidates"]


@pytest.mark.parametrize("case", GRAPH_CASES, ids=CASE_IDS)
def test_scores_match_reference_bitwise_on_cpu(case):
    rec = RECORDS[case.name]
    model, req = build_model(gm, case), build_request(gm, case)
    q, cands = _banks(model, req)
    raw = model.score(q, cands, device="cpu")
    assert raw.view(torch.int32).tolist() == rec["raw_scores"]
    tok = gm.graph_mneme_request_token_scores(case.seq_len, req, model=model, device="cpu")
    assert _digest(tok.numpy()) == rec["token_scores"]["digest"]
    assert torch.unique(tok).view(torch.int32).tolist() == rec["token_scores"]["unique"]


def test_graph_scores_select_like_the_reference():
    """Chunk-level scores tie at both selection boundaries; the oracle's
    restatement of torch's CPU topk order reproduces the reference's lists."""
    case = next(c for c in GRAPH_CASES if c.cache)
    rec = RECORDS[case.name]["cache"]
    assert rec["ties"] == {"protect": True, "cold": True}
    model, req = build_model(gm, case), build_request(gm, case)
    tok = gm.graph_mneme_request_token_scores(case.seq_len, req, model=model, device="cpu").numpy()
    pol = orc.POLICIES[rec["profile"]]
    ret, std, cold = orc.select_tiers(case.seq_len, pol, tok)
    for layer in rec["layers"]:
        assert ret.tolist() == layer["idx_ret"]
        assert _digest(std) == layer["idx_std_digest"] and std.size == layer["n_std"]
        assert _digest(cold) == layer["idx_cold_digest"] and cold.size == layer["n_cold"]


def test_normalize_modes_and_errors():
    s = torch.tensor([3.0, 1.0, 2.0])
    assert gm.normalize_graph_scores(s, mode="minmax").tolist() == [1.0, 0.0, 0.5]
    assert gm.normalize_graph_scores(torch.full((3,), 2.0), mode="minmax").tolist() == [1.0, 1.0, 1.0]
    assert gm.normalize_graph_scores(torch.full((3,), 2.0), mode="zscore").tolist() == [0.0, 0.0, 0.0]
    assert gm.normalize_graph_scores(s, mode="none") is not None
    with pytest.raises(ValueError):
        gm.normalize_graph_scores(s, mode="rank")


def test_missing_bundled_weights_raise(monkeypatch, tmp_path):
    monkeypatch.setenv("GRAPHKV_MNEME_WEIGHTS", str(tmp_path / "absent.safetensors"))
    with pytest.raises(FileNotFoundError):
        gm.load_bundled_graph_model("cpu")


def test_user_weights_load_from_safetensors(monkeypatch, tmp_path):
    from safetensors.torch import save_file

    case = next(c for c in GRAPH_CASES if not c.geometry)
    model = build_model(gm, case)
    path = tmp_path / "latest.safetensors"
    save_file({k: v.contiguous() for k, v in model.state_dict().items()}, str(path))
    monkeypatch.setenv("GRAPHKV_MNEME_WEIGHTS", str(path))
    loaded = gm.load_bundled_graph_model("cpu")
    for k, v in model.state_dict().items():
        assert torch.equal(loaded.state_dict()[k], v)


@pytest.mark.gpu
def test_graph_memory_request_on_gpu_matches_reference():
    """quantize_hf_cache(graph_memory=request) with the scorer and the whole
    compression on the GPU: same index lists and stats as the reference."""
    from graphkv_b200 import quantize_hf_cache
    from graphkv_b200 import _lib as L

    case = next(c for c in GRAPH_CASES if c.cache)
    rec = RECORDS[case.name]["cache"]
    model, req = build_model(gm, case), build_request(gm, case)
    layers = tuple((k.cuda(), v.cuda()) for k, v in cache_layers(case))
    comp = quantize_hf_cache(layers, rec["profile"], graph_memory=req, graph_mneme_model=model,
                             graph_mneme_device="cuda", output="compressed")
    torch.cuda.synchronize()
    assert L.device_error() == 0
    for ql, ref in zip(comp.layers, rec["layers"]):
        assert ql.retained_indices.cpu().tolist() == ref["idx_ret"]
        assert _digest(ql.compressed_indices.cpu().numpy()) == ref["idx_std_digest"]
        assert _digest(ql.low_priority_compressed_indices.cpu().numpy()) == ref["idx_cold_digest"]
    assert comp.stats() == rec["stats"]
