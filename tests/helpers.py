"""Shared helpers of the parity tests."""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import torch

from graphkv_b200 import KvQuantConfig, get_profile
from tests.golden.cases import bits_of

SCALE_DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def config_for(case) -> KvQuantConfig:
    cfg = get_profile(case.profile).config
    over = dict(case.overrides)
    if "scale_dtype" in over:
        over["scale_dtype"] = SCALE_DTYPES[over["scale_dtype"]]
    return replace(cfg, **over) if over else cfg


def layer_arrays(layer) -> dict:
    """Stored arrays of one QuantizedKvLayer in storage form (numpy, CPU)."""
    if layer.passthrough_keys is not None:
        return {"pass_k": bits_of(layer.passthrough_keys), "pass_v": bits_of(layer.passthrough_values)}
    out = {
        "idx_ret": layer.retained_indices.cpu().numpy(),
        "idx_std": layer.compressed_indices.cpu().numpy(),
        "idx_cold": (layer.low_priority_compressed_indices.cpu().numpy()
                     if layer.low_priority_compressed_indices is not None else np.zeros(0, np.int32)),
        "ret_k": bits_of(layer.retained_keys),
        "ret_v": bits_of(layer.retained_values),
    }
    for name, t in (("std_k", layer.compressed_keys), ("std_v", layer.compressed_values),
                    ("cold_k", layer.low_priority_compressed_keys), ("cold_v", layer.low_priority_compressed_values)):
        if t is None:
            continue
        out[name + ".q"] = t.q.cpu().numpy()
        out[name + ".scales"] = bits_of(t.scales)
        if t.zero_points is not None:
            out[name + ".zp"] = t.zero_points.cpu().numpy()
    return out
