"""The public API on the GPU: HF cache in/out, host-resident inputs, the
stand-alone tensor dequantize, append, and error reporting."""
import numpy as np
import pytest
import torch

import graphkv_b200 as g
from graphkv_b200 import _lib as L
from graphkv_b200.workloads import WORKLOADS, make_layer, make_scores
from oracle import graphkv_oracle as orc
from tests.golden.cases import bits_of

pytestmark = pytest.mark.gpu


def _small_cache(T=2048, layers=3, dtype=torch.bfloat16, device="cuda"):
    g_ = torch.Generator().manual_seed(5)
    return tuple((torch.randn(1, 2, T, 128, generator=g_).to(dtype).to(device),
                  torch.randn(1, 2, T, 128, generator=g_).to(dtype).to(device)) for _ in range(layers))


def test_dynamic_cache_export_matches_dequantize():
    from transformers.cache_utils import DynamicCache
    cache = _small_cache()
    scores = torch.exp(torch.randn(2048, generator=torch.Generator().manual_seed(1))).cuda()
    dyn = g.quantize_hf_cache(cache, "graphkv", importance_scores=scores, output="dynamic")
    comp = g.quantize_hf_cache(cache, "graphkv", importance_scores=scores, output="compressed")
    assert isinstance(dyn, DynamicCache)
    for i, (k, v) in enumerate(comp.dequantize()):
        assert torch.equal(dyn.layers[i].keys, k) and torch.equal(dyn.layers[i].values, v)
    assert dyn.get_seq_length() == 2048
    # an HF cache goes back in
    again = g.quantize_hf_cache(dyn, "graphkv-int4-balanced", output="compressed")
    assert again.stats()["layers"] == 3.0


def test_host_inputs_round_trip_to_host():
    cache = _small_cache(device="cpu")
    out = g.quantize_hf_cache(cache, "graphkv-int4-balanced", output="legacy")
    dev = g.quantize_hf_cache(tuple((k.cuda(), v.cuda()) for k, v in cache), "graphkv-int4-balanced",
                              output="legacy")
    for (hk, hv), (dk, dv) in zip(out, dev):
        assert hk.device.type == "cpu"
        assert torch.equal(hk, dk.cpu()) and torch.equal(hv, dv.cpu())


def test_quantized_tensor_dequantize_matches_oracle():
    cache = _small_cache(T=512, layers=1)
    cfg = g.get_profile("graphkv-int4-balanced").config
    layer = g.quantize_kv_layer(*cache[0], cfg)
    k = layer.compressed_keys.dequantize()
    K = cache[0][0].float().cpu().numpy()
    qt = orc.quantize_tensor(K, "bf16", 4, 64, "symmetric", 2)
    assert np.array_equal(bits_of(k), orc.storage_bits(orc.dequantize_tensor(qt), "bf16"))


def test_append_requantizes():
    cache = _small_cache(T=512, layers=2)
    cfg = g.get_profile("graphkv-int4-balanced").config
    comp = g.QuantizedKvCache.from_past_key_values(cache, cfg)
    new = tuple((torch.randn(1, 2, 64, 128, device="cuda").bfloat16(),
                 torch.randn(1, 2, 64, 128, device="cuda").bfloat16()) for _ in range(2))
    grown = comp.append(new, cfg)
    assert grown.layers[0].original_shape == (1, 2, 576, 128)
    k, v = grown.layers[1].dequantize()
    assert k.shape == (1, 2, 576, 128)


def test_reference_shaped_workload_stats():
    w = WORKLOADS["qwen7b-16k"]
    layers = [make_layer(w, l, device="cuda") for l in range(2)]
    comp = g.quantize_hf_cache(tuple(layers), "graphkv", importance_scores=make_scores(w, "cuda"),
                               output="compressed")
    st = comp.stats()
    assert st["compressed_bytes"] == 2 * 255_437_952 // 28
    assert st["low_priority_tokens"] == 2 * 3992 * 1


def test_bad_index_is_reported_not_faulted():
    """A caller-supplied index outside [0, T) is skipped and reported through
    the device error word (the kernels check every gathered position)."""
    cache = _small_cache(T=256, layers=1)
    cfg = g.get_profile("graphkv-int4-balanced").config
    layer = g.quantize_kv_layer(*cache[0], cfg)
    assert L.device_error() == 0
    layer.compressed_indices[3] = 10_000
    layer.dequantize()
    assert L.device_error() == 3
    assert L.device_error() == 0


def test_static_export_follows_reference_behaviour():
    cache = _small_cache(T=256, layers=1)
    comp = g.quantize_hf_cache(cache, "graphkv-int4-balanced", output="compressed")
    with pytest.raises(ValueError, match="config is required"):
        comp.to_hf_cache("static")
    with pytest.raises(ValueError, match="implementation must be"):
        comp.to_hf_cache("paged")


def _pinned(cache):
    return tuple((k.pin_memory(), v.pin_memory()) for k, v in cache)


@pytest.mark.parametrize("chunk", [1, 2, 4])
def test_pinned_host_round_trip_pipeline_matches_two_step_path(chunk):
    """The pipelined host path (copies in both directions overlapping the kernels,
    one selection shared by every chunk) returns the same bytes as compressing
    and then dequantizing, for a cache whose cold tier is rotated (T = 32768)."""
    from graphkv_b200.core import roundtrip_host_cache
    from graphkv_b200.profiles import get_profile
    cache = _pinned(_small_cache(T=32768, layers=5, device="cpu"))
    scores = torch.exp(2.0 * torch.randn(32768, generator=torch.Generator().manual_seed(3)))
    cfg = get_profile("graphkv").config
    piped = roundtrip_host_cache(cache, cfg, scores, chunk_layers=chunk)
    assert piped is not None and len(piped) == 5
    two_step = g.QuantizedKvCache.from_past_key_values(cache, cfg, scores).dequantize()
    assert L.device_error() == 0
    for (pk, pv), (tk, tv) in zip(piped, two_step):
        assert pk.device.type == "cpu" and pk.is_pinned()
        assert torch.equal(pk, tk) and torch.equal(pv, tv)


def test_quantize_hf_cache_takes_the_pipeline_for_pinned_host_caches(monkeypatch):
    from graphkv_b200 import core
    calls = []
    real = core.roundtrip_host_cache

    def spy(*a, **k):
        out = real(*a, **k)
        calls.append(out is not None)
        return out

    monkeypatch.setattr("graphkv_b200.integrations.roundtrip_host_cache", spy)
    cache = _small_cache(device="cpu")
    pinned = _pinned(cache)
    scores = torch.exp(torch.randn(2048, generator=torch.Generator().manual_seed(1)))
    legacy = g.quantize_hf_cache(pinned, "graphkv", importance_scores=scores, output="legacy")
    dyn = g.quantize_hf_cache(pinned, "graphkv", importance_scores=scores, output="dynamic")
    plain = g.quantize_hf_cache(cache, "graphkv", importance_scores=scores, output="legacy")  # pageable
    assert calls == [True, True, False]
    for i, ((lk, lv), (qk, qv)) in enumerate(zip(legacy, plain)):
        assert torch.equal(lk, qk) and torch.equal(lv, qv)
        assert torch.equal(dyn.layers[i].keys, qk) and torch.equal(dyn.layers[i].values, qv)
    with pytest.raises(ValueError, match="config is required"):
        g.quantize_hf_cache(pinned, "graphkv", importance_scores=scores, output="static")
    with pytest.raises(ValueError, match="implementation must be"):
        g.quantize_hf_cache(pinned, "graphkv", importance_scores=scores, output="paged")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tensors_on_another_gpu_than_the_current_one():
    """Every call runs on the GPU that holds its tensors, whichever GPU is
    current: cache on cuda:1 with cuda:0 current gives the same bytes as on cuda:0."""
    cache0 = _small_cache(T=16384, layers=2)  # long enough for a cold tier
    scores = torch.exp(torch.randn(4, 16384, generator=torch.Generator().manual_seed(2)))
    torch.cuda.set_device(0)
    ref = g.quantize_hf_cache(cache0, "graphkv", importance_scores=scores.cuda(0), output="compressed")
    cache1 = tuple((k.to("cuda:1"), v.to("cuda:1")) for k, v in cache0)
    other = g.quantize_hf_cache(cache1, "graphkv", importance_scores=scores.cuda(1), output="compressed")
    assert torch.cuda.current_device() == 0
    for la, lb in zip(ref.layers, other.layers):
        assert lb.compressed_keys.q.device == torch.device("cuda:1")
        assert torch.equal(la.retained_indices.cpu(), lb.retained_indices.cpu())
        assert torch.equal(la.compressed_keys.q.cpu(), lb.compressed_keys.q.cpu())
        assert la.low_priority_compressed_values is not None
        assert torch.equal(la.low_priority_compressed_values.q.cpu(), lb.low_priority_compressed_values.q.cpu())
    for (ka, va), (kb, vb) in zip(ref.dequantize(), other.dequantize()):
        assert kb.device == torch.device("cuda:1")
        assert torch.equal(ka.cpu(), kb.cpu()) and torch.equal(va.cpu(), vb.cpu())
    host = g.quantize_hf_cache(tuple((k.cpu(), v.cpu()) for k, v in cache1), "graphkv-int4-balanced",
                               output="legacy")
    assert host[0][0].device.type == "cpu"
    with torch.cuda.device(1):
        assert L.device_error() == 0
    assert L.device_error() == 0


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_pieces_rebuild_the_whole_cache(world):
    """Every rank's ShardedKvCache (built here in one process, one after the
    other) dequantizes to its slice of the unsharded result, and the summed
    per-layer counters give exactly the unsharded stats()."""
    from graphkv_b200.sharding import ShardedKvCache, shard_units, stats_from_rows

    cache = _small_cache(T=8192, layers=3)
    scores = torch.exp(2 * torch.randn(8192, generator=torch.Generator().manual_seed(4))).cuda()
    cfg = g.get_profile("graphkv").config
    whole = g.QuantizedKvCache.from_past_key_values(cache, cfg, scores)
    whole_deq = whole.dequantize()
    rows = 0
    for rank in range(world):
        units = shard_units(3, 2, world, rank)
        pieces = [(cache[l][0][:, h0:h1], cache[l][1][:, h0:h1]) for l, h0, h1 in units]
        sh = ShardedKvCache.from_past_key_values(pieces, units, 3, 2, cfg, scores)
        rows = rows + sh.stat_rows()
        for (k, v), (l, h0, h1) in zip(sh.dequantize(), units):
            assert torch.equal(k, whole_deq[l][0][:, h0:h1]) and torch.equal(v, whole_deq[l][1][:, h0:h1])
    assert stats_from_rows(rows) == whole.stats()
    assert L.device_error() == 0
