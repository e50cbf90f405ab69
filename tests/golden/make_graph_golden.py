"""Record the reference's Graph Mneme outputs for ``graph_cases.py``.

Run where the reference package is importable (pure Python, CPU):

    python tests/golden/make_graph_golden.py --src <reference>/src

For each case: the scorer's parameter names and shapes, the query/candidate
fact banks (``graph_model.py:362-422``), the raw chunk scores of
``GraphMemory17L.score`` (``graph_model.py:182-201``) as fp32 bit patterns,
the token scores of ``graph_mneme_request_token_scores``
(``graph_model.py:315-334``), and for cases with a cache the index lists that
``quantize_hf_cache(..., graph_memory=request)`` selects
(``integrations.py:40-52``), plus whether a selection boundary falls inside a
run of equal scores.  Writes ``graph_mneme.json`` next to this file.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from math import ceil

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.graph_cases import GRAPH_CASES, build_model, build_request, cache_layers  # noqa: E402


def f32_bits(t: torch.Tensor) -> list[int]:
    return t.detach().to(torch.float32).contiguous().view(torch.int32).flatten().tolist()


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bank_record(bank) -> dict:
    return {"src": bank.src.tolist(), "rel": bank.rel.tolist(), "dst": bank.dst.tolist(),
            "entity_map": sorted(bank.entity_map.items()), "relation_map": sorted(bank.relation_map.items())}


def boundary_tie(values: torch.Tensor, keep: int, largest: bool) -> bool:
    if not 0 < keep < values.numel():
        return False
    v = torch.sort(values, descending=largest).values
    return bool(v[keep - 1] == v[keep])


def run(ref_pkg, gm, c) -> dict:
    model = build_model(gm, c)
    req = build_request(gm, c)
    cfg = model.cfg
    query = gm.build_query_bank(req.query_anchor, req.query_relation, req.query_facts, cfg,
                                shuffle_seed=req.shuffle_seed)
    cands = [gm.build_candidate_bank(ch.anchor, ch.facts, cfg, shuffle_seed=ch.shuffle_seed) for ch in req.chunks]
    raw = model.score(query, cands, device="cpu")
    tok = gm.graph_mneme_request_token_scores(c.seq_len, req, model=model, device="cpu")
    rec = {
        "case": c.name,
        "params": sorted((k, list(v.shape)) for k, v in model.state_dict().items()),
        "query": bank_record(query.facts), "query_relation": query.query_relation,
        "candidates": [bank_record(b) for b in cands],
        "raw_scores": f32_bits(raw),
        "token_scores": {"digest": digest(tok.numpy()), "unique": f32_bits(torch.unique(tok))},
    }
    if c.cache:
        profile = c.cache[0]
        layers = tuple(cache_layers(c))
        comp = ref_pkg.quantize_hf_cache(layers, profile, graph_memory=req, graph_mneme_model=model,
                                         graph_mneme_device="cpu", output="compressed")
        pcfg = ref_pkg.get_profile(profile).config
        sel = []
        for ql in comp.layers:
            sel.append({
                "idx_ret": ql.retained_indices.tolist(),
                "idx_std_digest": digest(ql.compressed_indices.numpy()),
                "n_std": int(ql.compressed_indices.numel()),
                "idx_cold_digest": digest(ql.low_priority_compressed_indices.numpy())
                if ql.low_priority_compressed_indices is not None else None,
                "n_cold": int(ql.low_priority_compressed_indices.numel())
                if ql.low_priority_compressed_indices is not None else 0,
            })
        # boundary ties of the two score selections
        from graphkv import core as ref_core
        base = ref_core.build_retention_mask(c.seq_len, pcfg, None)
        cand = (~base).nonzero().flatten()
        n = cand.numel()
        keep = min(n, max(ceil(n * pcfg.semantic_protection_ratio), pcfg.min_protected_tokens))
        protect_tie = boundary_tie(tok[cand], keep, True)
        mask = ref_core.build_retention_mask(c.seq_len, pcfg, tok)
        rest = (~mask).nonzero().flatten()
        ratio = ref_core._effective_low_priority_ratio(pcfg, c.seq_len)
        k_cold = min(rest.numel(), max(ceil(rest.numel() * ratio), pcfg.min_low_priority_tokens))
        cold_tie = boundary_tie(tok[rest], k_cold, False)
        rec["cache"] = {"profile": profile, "layers": sel, "stats": comp.stats(),
                        "ties": {"protect": protect_tie, "cold": cold_tie}}
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", required=True, help="the reference package's src directory (holds graphkv/)")
    args = ap.parse_args()
    sys.path.insert(0, args.src)
    import graphkv as ref_pkg
    from graphkv import graph_model as gm
    torch.manual_seed(0)
    out = {"reference": {"torch": torch.__version__, "graphkv": ref_pkg.__version__},
           "cases": [run(ref_pkg, gm, c) for c in GRAPH_CASES]}
    with open(os.path.join(HERE, "graph_mneme.json"), "w") as f:
        json.dump(out, f, indent=None, separators=(",", ":"), sort_keys=True)
    for c in out["cases"]:
        print(c["case"], len(c["raw_scores"]), c.get("cache", {}).get("ties"))


if __name__ == "__main__":
    main()
