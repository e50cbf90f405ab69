"""Large quantize / dequant calls run their rotated-tier launch on a
library-owned second stream, forked from and joined back into the caller's
stream.  Two host threads compressing and dequantizing different caches at the
same time, each on its own CUDA stream, must get exactly what one thread gets
doing the same work alone (integer codes, scales and dequantized bits: exact
equality).  The caches are large enough for the side stream (at least 8192
tiles) and long enough (32k tokens) for the rotated int2 cold tier."""
import threading

import numpy as np
import pytest
import torch

import graphkv_b200 as g
from graphkv_b200 import _lib as L
from tests.golden.cases import bits_of
from tests.helpers import layer_arrays

pytestmark = pytest.mark.gpu


def _cache(seed, layers=4, H=4, T=32768, D=128):
    gen = torch.Generator().manual_seed(seed)
    pairs = []
    for _ in range(layers):
        k = (torch.randn(1, H, T, D, generator=gen) * torch.exp(torch.randn(H, 1, D, generator=gen)))
        v = torch.randn(1, H, T, D, generator=gen)
        pairs.append((k.to(torch.bfloat16).cuda(), v.to(torch.bfloat16).cuda()))
    scores = torch.exp(2 * torch.randn(T, generator=gen)).cuda()
    return pairs, scores


def _compress_and_back(pairs, scores, cfg):
    cache = g.QuantizedKvCache.from_past_key_values(pairs, cfg, scores)
    deq = cache.dequantize()
    return cache, deq


def _same(a, b):
    (ca, da), (cb, db) = a, b
    for la, lb in zip(ca.layers, cb.layers):
        ma, mb = layer_arrays(la), layer_arrays(lb)
        assert ma.keys() == mb.keys()
        for name in ma:
            assert np.array_equal(ma[name], mb[name]), name
    for (ka, va), (kb, vb) in zip(da, db):
        assert np.array_equal(bits_of(ka), bits_of(kb)) and np.array_equal(bits_of(va), bits_of(vb))


def test_concurrent_calls_match_one_thread():
    cfg = g.get_profile("graphkv").config
    inputs = [_cache(11), _cache(12)]
    alone = [_compress_and_back(p, s, cfg) for p, s in inputs]
    torch.cuda.synchronize()
    assert alone[0][0].layers[0].low_priority_compressed_values.rotation == "hadamard"
    for _ in range(3):
        results, errors = [None, None], []

        def work(i):
            try:
                st = torch.cuda.Stream()
                with torch.cuda.stream(st):
                    results[i] = _compress_and_back(*inputs[i], cfg)
                st.synchronize()
            except Exception as e:  # reported below
                errors.append(e)

        threads = [threading.Thread(target=work, args=(i,)) for i in range(2)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        assert not errors, errors
        torch.cuda.synchronize()
        for i in range(2):
            _same(results[i], alone[i])
    assert L.device_error() == 0
