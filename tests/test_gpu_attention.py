"""Attention over a compressed layer read from its packed codes
(gkv_attention, attention_from_quantized) against the reference's way of
computing it: attention_from_kv over the dequantized layer in fp32
(core.py:800-820).  The rows attended over are the same bits, so the results
differ only by fp32 summation order: the test bar is a relative error below
1e-5 of the output's norm and a cosine of at least 0.999999 (in fp64)."""
import pytest
import torch

import graphkv_b200 as g
from graphkv_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _layer(profile, T, D=128, H=2, B=1, dtype=torch.bfloat16, scores=True, seed=1, **over):
    from dataclasses import replace
    gen = torch.Generator().manual_seed(seed)
    k = (torch.randn(B, H, T, D, generator=gen) * torch.exp(torch.randn(H, 1, D, generator=gen))).to(dtype)
    v = torch.randn(B, H, T, D, generator=gen).to(dtype)
    s = torch.exp(2 * torch.randn(T, generator=gen)).cuda() if scores else None
    cfg = g.get_profile(profile).config
    cfg = replace(cfg, **over) if over else cfg
    return g.quantize_kv_layer(k.cuda(), v.cuda(), cfg, importance_scores=s)


def _check(layer, Q, seed=2):
    B, H, T, D = layer.original_shape
    q = torch.randn(B, H, Q, D, generator=torch.Generator().manual_seed(seed)).cuda()
    mine = g.attention_from_quantized(q, layer)
    keys, values = layer.dequantize()
    ref, _ = g.attention_from_kv(q, keys, values)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    a, b = mine.double().flatten(), ref.double().flatten()
    rel = float((a - b).norm() / b.norm())
    cos = float(torch.dot(a, b) / (a.norm() * b.norm()))
    assert rel < 1e-5 and cos >= 0.999999, (rel, cos)


@pytest.mark.parametrize("Q", [1, 4, 16])
def test_long_context_graphkv_layer(Q):
    """32k tokens: retained rows, int4 keys, int4 values and a Hadamard-rotated
    int2 cold tier, batch 2."""
    _check(_layer("graphkv", 32768, B=2), Q)


@pytest.mark.parametrize("profile,T,D,dtype", [
    ("graphkv", 8192, 128, torch.bfloat16),          # 25% cold tier, not rotated
    ("graphkv-int4-balanced", 4096, 64, torch.bfloat16),
    ("graphkv-qwen7-nf4", 2048, 128, torch.float16),  # affine, groups of 32
    ("graphkv-int4-balanced", 1000, 128, torch.float32),
])
def test_other_profiles_and_dtypes(profile, T, D, dtype):
    _check(_layer(profile, T, D=D, dtype=dtype, scores=profile == "graphkv"), 3)


def test_uncovered_layers_take_the_dequantized_path():
    """Keys grouped along channels and a passthrough layer: same results."""
    _check(_layer("graphkv-int4-balanced", 512, key_group_axis="channel", value_group_axis="token"), 2)
    _check(_layer("graphkv-int4-balanced", 16, D=8, bits=8, group_size=1, scores=False), 1)


def test_query_shape_errors():
    layer = _layer("graphkv-int4-balanced", 256, scores=False)
    with pytest.raises(ValueError, match="rank-4"):
        g.attention_from_quantized(torch.zeros(2, 1, 128).cuda(), layer)
    with pytest.raises(ValueError, match="batch/head/head_dim"):
        g.attention_from_quantized(torch.zeros(1, 3, 1, 128).cuda(), layer)
