"""Glue between torch tensors / golden cases and the numpy oracle (test helper)."""
from __future__ import annotations

import json
import os
from contextlib import contextmanager
from dataclasses import replace

import numpy as np
import torch

from oracle import graphkv_oracle as orc
from tests.golden.cases import tensor_digest

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TORCH_TO_TAG = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().to(torch.float32).numpy()


def policy_for(case) -> orc.Policy:
    return replace(orc.POLICIES[case.profile], **case.overrides) if case.overrides else orc.POLICIES[case.profile]


def scores_np(scores):
    if scores is None:
        return None
    if isinstance(scores, (list, tuple)):
        return [to_np(s) for s in scores]
    return to_np(scores)


def oracle_layers(case, layers, scores):
    p = policy_for(case)
    out = []
    for li, (k, v) in enumerate(layers):
        s = scores[li] if isinstance(scores, list) else scores
        out.append(orc.quantize_layer(to_np(k), to_np(v), TORCH_TO_TAG[k.dtype], p, s))
    return out


def oracle_arrays(ql: orc.QLayer) -> dict:
    if ql.passthrough is not None:
        return {"pass_k": orc.storage_bits(ql.passthrough[0], ql.dtype),
                "pass_v": orc.storage_bits(ql.passthrough[1], ql.dtype)}
    return orc.layer_tensors(ql)


def load_golden(name):
    with open(os.path.join(GOLDEN_DIR, name + ".json")) as f:
        rec = json.load(f)
    npz = os.path.join(GOLDEN_DIR, name + ".npz")
    arrays = dict(np.load(npz)) if os.path.exists(npz) else {}
    return rec, arrays


def compare_arrays(name, mine: dict, golden_layer: dict, golden_arrays: dict, li: int):
    """Return a list of mismatch descriptions between my stored arrays and the golden record."""
    problems = []
    gt = golden_layer["tensors"]
    if set(mine) != set(gt):
        problems.append(f"{name} l{li}: tensor set {sorted(mine)} != {sorted(gt)}")
    for n, a in mine.items():
        if n not in gt:
            continue
        if tensor_digest(a) != gt[n]["digest"]:
            key = f"l{li}.{n}"
            detail = ""
            if key in golden_arrays:
                g = golden_arrays[key]
                if g.shape == a.shape:
                    bad = np.nonzero(g.reshape(-1) != a.reshape(-1))[0]
                    detail = f" ({bad.size} of {g.size} differ, first at {bad[:5].tolist()})"
                else:
                    detail = f" (shape {a.shape} vs {g.shape})"
            problems.append(f"{name} l{li}: {n} digest mismatch dtype {a.dtype}/{gt[n]['dtype']}{detail}")
    return problems


@contextmanager
def reference_threads(rec: dict):
    """Run with the torch CPU thread count the golden was recorded with: it sets
    the column blocks of torch's CPU mean over score rows, which both the oracle
    and the library's score averaging follow."""
    n = int(rec.get("torch_threads", torch.get_num_threads()))
    old_torch, old_oracle = torch.get_num_threads(), orc.SUM_THREADS
    torch.set_num_threads(n)
    orc.SUM_THREADS = n
    try:
        yield n
    finally:
        torch.set_num_threads(old_torch)
        orc.SUM_THREADS = old_oracle
