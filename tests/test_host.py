"""Host-side logic that needs no GPU: config validation, profiles, cache
extraction, API errors, and that the compute path refuses to run without CUDA."""
from dataclasses import replace

import pytest
import torch

import graphkv_b200 as g
from graphkv_b200 import KvQuantConfig, get_profile, hf_cache_to_tuple


@pytest.mark.parametrize("field,value,msg", [
    ("bits", 3, "bits must be 2, 4, or 8"),
    ("key_bits", 5, "key_bits must be 2, 4, 8, or None."),
    ("group_size", 0, "group_size must be >= 1."),
    ("quantizer", "nf4", "quantizer must be 'symmetric' or 'affine'."),
    ("semantic_protection_ratio", 1.5, "semantic_protection_ratio must be in [0, 1]."),
    ("rotation", "dct", "rotation must be 'none' or 'hadamard'."),
    ("low_priority_value_bits", 3, "low_priority_value_bits must be 2, 4, 8, or None."),
    ("min_outlier_tokens", -1, "min_outlier_tokens must be >= 0."),
])
def test_validate_messages(field, value, msg):
    with pytest.raises(ValueError, match=msg.replace("(", r"\(").replace(")", r"\)").replace("[", r"\[")):
        replace(KvQuantConfig(), **{field: value}).validate()


def test_profiles():
    assert get_profile("graphkv").config.low_priority_value_rotation == "hadamard"
    p = get_profile("graphkv-int4-balanced")
    assert get_profile(p) is p
    with pytest.raises(KeyError, match="Unknown GraphKV profile"):
        get_profile("nope")
    assert len(g.list_profiles()) == 9
    with pytest.raises(ValueError, match="engine-native recipe"):
        g.quantize_hf_cache(((torch.zeros(1, 1, 4, 8), torch.zeros(1, 1, 4, 8)),), "vllm-fp8")


def test_hf_cache_to_tuple_forms():
    k = torch.randn(1, 2, 5, 8)
    v = torch.randn(1, 2, 5, 8)
    assert hf_cache_to_tuple(((k, v), None, (k, v)))[1][0] is k
    from transformers.cache_utils import DynamicCache
    c = DynamicCache()
    c.update(k, v, 0)
    (k2, v2), = hf_cache_to_tuple(c)
    assert torch.equal(k2, k)
    with pytest.raises(TypeError, match="Unsupported cache type"):
        hf_cache_to_tuple(object())
    with pytest.raises(TypeError, match="Legacy cache layers"):
        hf_cache_to_tuple([(k,)])


def test_shape_errors_precede_any_compute():
    cfg = get_profile("graphkv").config
    with pytest.raises(ValueError, match="same shape"):
        g.quantize_kv_layer(torch.zeros(1, 1, 4, 8), torch.zeros(1, 1, 5, 8), cfg)
    with pytest.raises(ValueError, match="batch, heads, tokens, head_dim"):
        g.quantize_kv_layer(torch.zeros(1, 4, 8), torch.zeros(1, 4, 8), cfg)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    cfg = get_profile("graphkv-int4-balanced").config
    with pytest.raises(RuntimeError, match="CUDA device"):
        g.quantize_kv_layer(torch.randn(1, 1, 256, 64), torch.randn(1, 1, 256, 64), cfg)


def _fastdiv(d):
    """Host constants of the tile kernels' invariant-divisor division (Granlund and
    Montgomery, PLDI 1994, figure 4.1), restated: m = floor(2^32 (2^l - d) / d) + 1."""
    l = (d - 1).bit_length()
    return ((1 << 32) * ((1 << l) - d)) // d + 1, (1 if l > 0 else 0), (l - 1 if l > 0 else 0)


def test_invariant_divisor_division_is_exact():
    import random
    rng = random.Random(5)
    divisors = [1, 2, 3, 5, 7, 64, 112, 253, 1000, 4096, 65535, 2 ** 31 - 1, 2 ** 31]
    divisors += [rng.randrange(1, 2 ** 31) for _ in range(200)]
    for d in divisors:
        m, s1, s2 = _fastdiv(d)
        assert 0 <= m < 2 ** 32
        nums = [0, 1, d - 1, d, d + 1, 2 ** 32 - 1, 2 ** 32 - 2, 2 ** 31] + [rng.randrange(2 ** 32) for _ in range(300)]
        for n in nums:
            t = (m * n) >> 32
            assert (t + ((n - t) >> s1)) >> s2 == n // d, (d, n)
