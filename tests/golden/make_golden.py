"""Record the reference's own outputs for the golden cases.

Run in a container where the reference package is importable (pure Python):

    python tests/golden/make_golden.py --src <reference>/src [--only NAME ...]

For every case in ``cases.py`` this imports the reference ``graphkv`` package,
runs ``quantize_kv_layer`` (``core.py:647-772``) layer by layer on the seeded
CPU inputs, then ``dequantize`` (``core.py:265-307``), and writes

* ``<case>.json``: input digests, every stored tensor's digest/dtype/shape,
  tensor metadata (bits, group size, padding, q_shape ...), dequantized K/V
  digests, ``stats()`` and ``layer_stats()``, and boundary-tie flags;
* ``<case>.npz`` (small cases only): the stored arrays themselves (codes,
  scale bit patterns, zero points, index lists, retained rows) up to 64 KiB each.

The generated files are committed; the tests only read them.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from dataclasses import replace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.cases import CASES, bits_of, case_layers, case_scores, tensor_digest  # noqa: E402

MAX_ARRAY_BYTES = 64 * 1024
SCALE_DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def ref_config(ref, case):
    cfg = ref.get_profile(case.profile).config
    over = dict(case.overrides)
    if "scale_dtype" in over:
        over["scale_dtype"] = SCALE_DTYPES[over["scale_dtype"]]
    return replace(cfg, **over) if over else cfg


def ref_layer_arrays(layer):
    """Stored arrays of one reference QuantizedKvLayer in storage form."""
    out, meta = {}, {}
    if layer.passthrough_keys is not None:
        out["pass_k"] = bits_of(layer.passthrough_keys)
        out["pass_v"] = bits_of(layer.passthrough_values)
        return out, {"passthrough": True}
    out["idx_ret"] = layer.retained_indices.numpy()
    out["idx_std"] = layer.compressed_indices.numpy()
    lp = layer.low_priority_compressed_indices
    out["idx_cold"] = lp.numpy() if lp is not None else np.zeros(0, np.int32)
    out["ret_k"] = bits_of(layer.retained_keys)
    out["ret_v"] = bits_of(layer.retained_values)
    for name, t in (("std_k", layer.compressed_keys), ("std_v", layer.compressed_values),
                    ("cold_k", layer.low_priority_compressed_keys), ("cold_v", layer.low_priority_compressed_values)):
        if t is None:
            continue
        out[name + ".q"] = t.q.numpy()
        out[name + ".scales"] = bits_of(t.scales)
        if t.zero_points is not None:
            out[name + ".zp"] = t.zero_points.numpy()
        meta[name] = {"bits": t.bits, "group_size": t.group_size, "padded": t.padded, "q_shape": list(t.q_shape),
                      "packed": t.packed, "packed_offset": t.packed_offset, "rotation": t.rotation, "axis": t.axis,
                      "scales_shape": list(t.scales.shape), "q_dtype": str(t.q.dtype)}
    meta["passthrough"] = False
    return out, meta


def boundary_ties(ref_core, T, cfg, scores):
    """Whether the protection boundary falls inside a run of equal scores."""
    if scores is None or isinstance(scores, (list, tuple)):
        return {}
    s = ref_core._normalize_token_scores(T, scores, torch.device("cpu"))
    res = {}
    mask = ref_core.build_retention_mask(T, cfg, None)
    cand = (~mask).nonzero().flatten()
    if T >= cfg.semantic_protection_min_context and cand.numel():
        n = cand.numel()
        keep = min(n, max(int(np.ceil(n * cfg.semantic_protection_ratio)), cfg.min_protected_tokens))
        v = torch.sort(s[cand], descending=True).values
        res["protect"] = bool(0 < keep < n and v[keep - 1] == v[keep])
    return res


def run_case(ref, ref_core, case):
    t0 = time.time()
    cfg = ref_config(ref, case)
    layers = case_layers(case)
    scores = case_scores(case)
    rec = {"case": case.name, "profile": case.profile, "overrides": case.overrides,
           "reference": {"torch": torch.__version__, "graphkv": ref.__version__}, "layers": []}
    arrays = {}
    qlayers = []
    for li, (k, v) in enumerate(layers):
        s = scores[li] if isinstance(scores, list) else scores
        ql = ref_core.quantize_kv_layer(k, v, cfg, importance_scores=s)
        qlayers.append(ql)
        arrs, meta = ref_layer_arrays(ql)
        dk, dv = ql.dequantize()
        entry = {
            "inputs": {"k": tensor_digest(bits_of(k)), "v": tensor_digest(bits_of(v))},
            "tensors": {n: {"digest": tensor_digest(a), "dtype": str(a.dtype), "shape": list(a.shape)}
                        for n, a in arrs.items()},
            "meta": meta,
            "dequant": {"k": tensor_digest(bits_of(dk)), "v": tensor_digest(bits_of(dv))},
            "layer_stats": ql.stats(),
            "memory_bytes": ql.memory_bytes(),
        }
        rec["layers"].append(entry)
        if case.full_arrays:
            for n, a in arrs.items():
                if a.nbytes <= MAX_ARRAY_BYTES:
                    arrays[f"l{li}.{n}"] = a
            for n, a in (("deq_k", bits_of(dk)), ("deq_v", bits_of(dv))):
                if a.nbytes <= MAX_ARRAY_BYTES:
                    arrays[f"l{li}.{n}"] = a
        del dk, dv
    cache = ref_core.QuantizedKvCache(qlayers)
    rec["stats"] = cache.stats()
    T = layers[0][0].shape[2]
    rec["ties"] = boundary_ties(ref_core, T, cfg, scores)
    rec["torch_threads"] = torch.get_num_threads()  # sets the column blocks of a CPU mean over rows
    if isinstance(scores, torch.Tensor) and scores.numel() != T:
        mean_bits = bits_of(ref_core._normalize_token_scores(T, scores, torch.device("cpu")))
        rec["score_mean"] = tensor_digest(mean_bits)
        arrays["score_mean"] = mean_bits
    rec["seconds"] = round(time.time() - t0, 2)
    return rec, arrays


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", required=True, help="the reference package's src directory (holds graphkv/)")
    ap.add_argument("--only", nargs="*")
    ap.add_argument("--small", action="store_true", help="only the small (non-workload) cases")
    args = ap.parse_args()
    sys.path.insert(0, args.src)
    import graphkv as ref
    from graphkv import core as ref_core
    torch.set_num_threads(os.cpu_count() or 1)
    for case in CASES:
        if args.only and case.name not in args.only:
            continue
        if args.small and case.workload:
            continue
        rec, arrays = run_case(ref, ref_core, case)
        with open(os.path.join(HERE, case.name + ".json"), "w") as f:
            json.dump(rec, f, indent=1, sort_keys=True)
        npz = os.path.join(HERE, case.name + ".npz")
        if arrays:
            np.savez_compressed(npz, **arrays)
        elif os.path.exists(npz):
            os.remove(npz)
        print(f"{case.name}: {rec['seconds']} s, {len(arrays)} arrays", flush=True)


if __name__ == "__main__":
    main()
