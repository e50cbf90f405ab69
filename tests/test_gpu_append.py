"""Streaming append on the GPU (reference core.py:325-348, 418-433): the old
tokens are dequantized straight into the grown buffers and requantized with
the new ones.  The result must be the reference's -- requantize(cat(dequantize
(old), new)) -- byte for byte: checked against the numpy oracle's restatement
of that chain and against the library's own compress of the concatenated
cache."""
import numpy as np
import pytest
import torch

import graphkv_b200 as g
from graphkv_b200 import _lib as L
from oracle import graphkv_oracle as orc
from tests.golden.cases import bits_of
from tests.helpers import layer_arrays
from tests.oracle_bridge import oracle_arrays

pytestmark = pytest.mark.gpu


def _cache(T, layers=2, D=128, H=2, dtype=torch.bfloat16, seed=3):
    gen = torch.Generator().manual_seed(seed)
    return [((torch.randn(1, H, T, D, generator=gen) * torch.exp(torch.randn(H, 1, D, generator=gen))).to(dtype),
             torch.randn(1, H, T, D, generator=gen).to(dtype)) for _ in range(layers)]


def _same_layers(a, b):
    for la, lb in zip(a.layers, b.layers):
        ma, mb = layer_arrays(la), layer_arrays(lb)
        assert ma.keys() == mb.keys()
        for name in ma:
            assert np.array_equal(ma[name], mb[name]), name
    assert a.stats() == b.stats()


@pytest.mark.parametrize("n", [1, 200])
def test_append_matches_reference_chain(n):
    T, profile = 8192, "graphkv"
    cfg = g.get_profile(profile).config
    old = _cache(T)
    new = _cache(n, seed=9)
    gen = torch.Generator().manual_seed(5)
    s_old = torch.exp(2 * torch.randn(T, generator=gen))
    s_new = torch.exp(2 * torch.randn(T + n, generator=gen))
    cache = g.QuantizedKvCache.from_past_key_values([(k.cuda(), v.cuda()) for k, v in old], cfg, s_old.cuda())
    grown = cache.append([(k.cuda(), v.cuda()) for k, v in new], cfg, s_new.cuda())
    torch.cuda.synchronize()
    assert L.device_error() == 0
    # the library's own two-step chain
    deq = cache.dequantize()
    cat = [(torch.cat([dk, nk.cuda()], 2), torch.cat([dv, nv.cuda()], 2)) for (dk, dv), (nk, nv) in zip(deq, new)]
    _same_layers(grown, g.QuantizedKvCache.from_past_key_values(cat, cfg, s_new.cuda()))
    # the reference's chain, restated by the oracle
    pol = orc.POLICIES[profile]
    for li, ((k, v), (nk, nv)) in enumerate(zip(old, new)):
        ql = orc.quantize_layer(k.float().numpy(), v.float().numpy(), "bf16", pol, s_old.numpy())
        dk, dv = orc.dequantize_layer(ql)
        K = np.concatenate([dk, nk.float().numpy()], axis=2)
        V = np.concatenate([dv, nv.float().numpy()], axis=2)
        ref = orc.quantize_layer(K, V, "bf16", pol, s_new.numpy())
        mine, theirs = layer_arrays(grown.layers[li]), oracle_arrays(ref)
        for name in theirs:
            assert np.array_equal(mine[name].reshape(-1), theirs[name].reshape(-1)), (li, name)
        assert grown.layers[li].memory_bytes() == ref.memory_bytes()


def test_append_unaligned_rows_and_single_layer():
    """head_dim 40 (no tile kernels; grown slices of odd length are not 16-byte
    aligned) and QuantizedKvLayer.append."""
    cfg = g.get_profile("graphkv-int4-balanced").config
    (k, v), = _cache(301, layers=1, D=40)
    (nk, nv), = _cache(6, layers=1, D=40, seed=4)
    layer = g.quantize_kv_layer(k.cuda(), v.cuda(), cfg)
    grown = layer.append(nk.cuda(), nv.cuda(), cfg)
    dk, dv = layer.dequantize()
    again = g.quantize_kv_layer(torch.cat([dk, nk.cuda()], 2), torch.cat([dv, nv.cuda()], 2), cfg)
    for name, a in layer_arrays(grown).items():
        assert np.array_equal(a, layer_arrays(again)[name]), name
    gk, gv = grown.dequantize()
    assert gk.shape == (1, 2, 307, 40)


def test_append_to_passthrough_and_host_layers():
    from dataclasses import replace
    cfg = replace(g.get_profile("graphkv-int4-balanced").config, bits=8, group_size=1)
    (k, v), = _cache(16, layers=1, D=8)
    (nk, nv), = _cache(3, layers=1, D=8, seed=6)
    cache = g.QuantizedKvCache.from_past_key_values([(k, v)], cfg)  # host inputs, passthrough layer
    grown = cache.append([(nk, nv)], cfg)
    gk, gv = grown.dequantize()[0]
    assert torch.equal(gk.cpu(), torch.cat([k, nk], 2)) and torch.equal(gv.cpu(), torch.cat([v, nv], 2))
    host = g.QuantizedKvCache.from_past_key_values(_cache(512, layers=1), g.get_profile("graphkv").config)
    hk, _ = host.append(_cache(5, layers=1, seed=8), g.get_profile("graphkv").config).dequantize()[0]
    assert hk.device.type == "cpu" and hk.shape[2] == 517


def test_append_shape_errors():
    cfg = g.get_profile("graphkv-int4-balanced").config
    cache = g.QuantizedKvCache.from_past_key_values([(k.cuda(), v.cuda()) for k, v in _cache(256, layers=1)], cfg)
    with pytest.raises(ValueError, match="one \\(key, value\\) pair per cached layer"):
        cache.append([], cfg)
    with pytest.raises(ValueError, match="batch/head"):
        cache.append([(torch.zeros(1, 3, 2, 128), torch.zeros(1, 3, 2, 128))], cfg)
    with pytest.raises(ValueError, match="head_dim"):
        cache.append([(torch.zeros(1, 2, 2, 64), torch.zeros(1, 2, 2, 64))], cfg)
    with pytest.raises(ValueError, match="same shape"):
        cache.append([(torch.zeros(1, 2, 2, 128), torch.zeros(1, 2, 3, 128))], cfg)
