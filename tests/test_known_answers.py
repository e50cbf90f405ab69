"""The reference's published byte totals (README.md:25-30, 125, 128, 131, 134):
data-independent functions of shape and policy, reproduced by the host-side
accounting that sizes every allocation before the kernels run."""
import numpy as np
import pytest
import torch

from graphkv_b200.config import resolve_tiers, tensor_plans, layer_memory_bytes
from graphkv_b200.profiles import get_profile
from oracle import graphkv_oracle as orc

KATS = [
    ("graphkv-qwen7-nf4", 1024, False, 43_352_064),
    ("graphkv-qwen7-nf4", 4096, False, 95_993_856),
    ("graphkv-qwen7-nf4", 16384, False, 292_454_400),
    ("graphkv-qwen7-nf4", 32768, False, 558_530_560),
    ("graphkv", 1024, False, 32_169_984),
    ("graphkv", 4096, False, 80_683_008),
    ("graphkv", 16384, True, 255_437_952),
    ("graphkv", 32768, True, 487_457_152),
]
ORIGINAL = {1024: 58_720_256, 4096: 234_881_024, 16384: 939_524_096, 32768: 1_879_048_192}


@pytest.mark.parametrize("profile,T,scores,expected", KATS)
def test_published_cache_bytes(profile, T, scores, expected):
    cfg = get_profile(profile).config
    shape = (1, 4, T, 128)  # Qwen2.5-7B: 28 layers x 4 kv-heads x head_dim 128, bf16
    tiers = resolve_tiers(cfg, T, scores)
    plans = tensor_plans(cfg, shape, tiers)
    assert 28 * layer_memory_bytes(shape, torch.bfloat16, tiers, plans) == expected
    assert 2 * 28 * 4 * T * 128 * 2 == ORIGINAL[T]


def test_oracle_reproduces_a_published_total():
    """One layer through the oracle on random data gives the same bytes (x 28)."""
    rng = np.random.default_rng(1)
    K = orc.round_to(rng.standard_normal((1, 4, 4096, 128)).astype(np.float32), "bf16")
    V = orc.round_to(rng.standard_normal((1, 4, 4096, 128)).astype(np.float32), "bf16")
    ql = orc.quantize_layer(K, V, "bf16", orc.POLICIES["graphkv-qwen7-nf4"])
    assert 28 * ql.memory_bytes() == 95_993_856


@pytest.mark.parametrize("profile", ["graphkv", "graphkv-int2-max", "graphkv-int4-balanced",
                                     "graphkv-qwen7-nf4", "graphkv-int4-safe"])
@pytest.mark.parametrize("T", [1, 5, 64, 700, 8192, 9000, 32768])
@pytest.mark.parametrize("scores", [False, True])
def test_tier_sizes_match_oracle(profile, T, scores):
    cfg = get_profile(profile).config
    s = np.exp(np.random.default_rng(T).standard_normal(T)).astype(np.float32) if scores else None
    K = np.random.default_rng(2).standard_normal((1, 1, T, 8)).astype(np.float32)
    r, c, l = orc.select_tiers(T, orc.POLICIES[profile], s, K, K)
    t = resolve_tiers(cfg, T, scores)
    assert (t.n_retained, t.n_standard, t.n_cold) == (r.size, c.size, l.size)
