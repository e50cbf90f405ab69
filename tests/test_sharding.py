"""Weak sharding by (layer, kv-head) and the all-gather of per-shard byte counts
(the multi-GPU path of the benchmark), run as two gloo ranks on the CPU."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from graphkv_b200 import get_profile
from graphkv_b200.sharding import combine_stats, shard_bytes, shard_stats, shard_units

GEOM = dict(layers=3, heads=4, batch=2, seq=9000, dim=64)


@pytest.mark.parametrize("layers,heads", [(1, 1), (3, 4), (28, 4), (5, 8)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_partition_the_units(layers, heads, world):
    seen = []
    for rank in range(world):
        for layer, h0, h1 in shard_units(layers, heads, world, rank):
            assert 0 <= layer < layers and 0 <= h0 < h1 <= heads
            seen.extend((layer, h) for h in range(h0, h1))
    assert sorted(seen) == [(l, h) for l in range(layers) for h in range(heads)]
    assert len(seen) == len(set(seen))


def _whole_cache_bytes(cfg):
    g = GEOM
    comp = orig = 0
    for _ in range(g["layers"]):
        c, o = shard_bytes((g["batch"], g["heads"], g["seq"], g["dim"]), torch.bfloat16, cfg, True, 0)
        comp, orig = comp + c, orig + o
    return comp, orig


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = get_profile("graphkv").config
        g = GEOM
        comp = orig = 0
        for layer, h0, h1 in shard_units(g["layers"], g["heads"], world, rank):
            c, o = shard_bytes((g["batch"], h1 - h0, g["seq"], g["dim"]), torch.bfloat16, cfg, True, h0)
            comp, orig = comp + c, orig + o
        gathered = torch.empty(world * 2, dtype=torch.float64)
        dist.all_gather_into_tensor(gathered, shard_stats(comp, orig))
        out[rank] = combine_stats(gathered)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gathered_shard_bytes_equal_the_whole_cache(world):
    port = 29400 + world + (os.getpid() % 200)
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        results = [out[r] for r in range(world)]
    comp, orig = _whole_cache_bytes(get_profile("graphkv").config)
    for r in results:  # every rank derives the same whole-cache statistics
        assert r["shards"] == world
        assert r["memory_bytes"] == comp and r["original_memory_bytes"] == orig
        assert r["compression_ratio"] == pytest.approx(orig / comp)
