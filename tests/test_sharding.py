"""Sharding by (layer, kv-head) unit and the one all-gather of per-layer counts
that rebuilds the whole cache's stats() (run as gloo ranks on the CPU).  The
single-process statistics the ranks must reproduce are the reference's own,
recorded for the 16k and 32k Qwen2.5-7B-shaped workloads."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from graphkv_b200 import get_profile
from graphkv_b200.sharding import (STAT_FIELDS, gather_stat_rows, planned_piece_row, shard_units,
                                   stats_from_rows)
from graphkv_b200.workloads import WORKLOADS
from tests.oracle_bridge import load_golden


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


def _rank_rows(wkey, world, rank, profile=None):
    w = WORKLOADS[wkey]
    cfg = get_profile(profile or w.profile).config
    rows = torch.zeros(w.layers, len(STAT_FIELDS), dtype=torch.int64)
    for layer, h0, h1 in shard_units(w.layers, w.heads, world, rank):
        piece = (w.batch, h1 - h0, w.seq, w.head_dim)
        rows[layer] += torch.tensor(planned_piece_row(piece, w.dtype, cfg, w.with_scores, h0, w.heads))
    return rows


def _rank(rank, world, port, wkey, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out[rank] = stats_from_rows(gather_stat_rows(_rank_rows(wkey, world, rank)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("wkey,golden", [("qwen7b-16k", "w_qwen7b_16k"), ("qwen7b-32k", "w_qwen7b_32k")])
@pytest.mark.parametrize("world", [2, 3])
def test_gathered_stats_equal_the_reference_stats(wkey, golden, world):
    port = 29400 + 7 * world + len(wkey) + (os.getpid() % 200)
    with mp.get_context("spawn").Manager() as m:  # no fork of a threaded process
        out = m.dict()
        mp.spawn(_rank, args=(world, port, wkey, out), nprocs=world, join=True)
        results = [out[r] for r in range(world)]
    rec, _ = load_golden(golden)
    for r in results:  # every rank rebuilds exactly the reference's 12 numbers
        assert r == rec["stats"]


@pytest.mark.parametrize("world", [1, 2, 4, 8, 5])
def test_planned_rows_of_any_split_sum_to_the_same_stats(world):
    whole = stats_from_rows(sum(_rank_rows("qwen7b-8x131k", 1, 0) for _ in range(1)))
    split = stats_from_rows(sum(_rank_rows("qwen7b-8x131k", world, r) for r in range(world)))
    assert split == whole
    assert whole["compressed_bytes"] == 15219853824.0 and whole["original_bytes"] == 60129542144.0


def test_passthrough_is_decided_on_the_whole_layer():
    """A layer that is not smaller as a whole stays passthrough in every piece,
    and its tokens are counted once."""
    cfg = get_profile("graphkv-int4-balanced").config
    from dataclasses import replace
    cfg = replace(cfg, bits=8, group_size=1)
    rows = [planned_piece_row((1, 1, 16, 8), torch.bfloat16, cfg, False, h, 2) for h in (0, 1)]
    assert rows[0] == [512, 512, 16, 0, 0] and rows[1] == [512, 512, 0, 0, 0]
    st = stats_from_rows(torch.tensor([[a + b for a, b in zip(*rows)]]))
    assert st["retained_tokens"] == 16.0 and st["compression_ratio"] == 1.0
