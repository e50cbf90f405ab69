"""Golden cases of the Graph Mneme scorer (``graph_memory=`` requests).

The reference ships no scorer weights, so each case fixes a scorer geometry
and fills every parameter from a seeded generator (``seeded_state_dict``); the
same function rebuilds the weights wherever the tests run, and only the
reference's outputs are stored (``graph_mneme.json``, written by
``make_graph_golden.py``).  Requests are built from seeded ``random.Random``
streams as plain tuples so that either package's request class can hold them.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field

import torch

SMALL = dict(num_entities=16, num_facts=8, num_cand_facts=6, num_candidates=8, num_relations=32, d_model=32,
             num_heads=4, encoder_layers=2, dropout=0.0)


@dataclass(frozen=True)
class GraphCase:
    name: str
    geometry: dict = field(default_factory=dict)   # GraphMemoryConfig overrides (empty = default geometry)
    seed: int = 1
    n_chunks: int = 6
    n_entities: int = 40        # global entity ids drawn from [0, n_entities)
    n_relations: int = 12
    query_facts: int = 10
    chunk_facts: int = 7
    seq_len: int = 1024
    normalize: str = "minmax"
    shuffle: bool = False
    unseen_query_relation: bool = False
    cache: tuple = ()           # (profile, B, H, D, layers): also record a quantize_hf_cache selection


GRAPH_CASES = [
    GraphCase("small_minmax", SMALL, seed=1),
    GraphCase("small_zscore", SMALL, seed=2, normalize="zscore"),
    GraphCase("small_none_shuffled", SMALL, seed=3, normalize="none", shuffle=True),
    GraphCase("small_overflow_slots", SMALL, seed=4, n_entities=60, n_relations=50, query_facts=20, chunk_facts=12),
    GraphCase("small_unseen_relation", SMALL, seed=5, unseen_query_relation=True),
    GraphCase("small_single_chunk", SMALL, seed=6, n_chunks=1),
    GraphCase("default_geometry", {}, seed=7, n_chunks=12, seq_len=16384,
              cache=("graphkv", 1, 2, 64, 2)),
]


def seeded_state_dict(shapes: dict[str, tuple], seed: int) -> dict[str, torch.Tensor]:
    """Deterministic values for every parameter: N(0, 0.25) from a generator
    seeded per parameter (sorted names); LayerNorm weights around 1."""
    out = {}
    for i, name in enumerate(sorted(shapes)):
        g = torch.Generator().manual_seed(seed * 1000 + i)
        t = torch.randn(shapes[name], generator=g) * 0.25
        if ("norm" in name) and name.endswith("weight"):
            t = 1.0 + 0.2 * t
        if name == "log_temp":
            t = 0.3 * t
        out[name] = t.contiguous()
    return out


def _facts(rng: random.Random, n: int, anchor: int, c: GraphCase) -> list[tuple[int, int, int]]:
    facts = []
    for _ in range(n):
        src = anchor if rng.random() < 0.4 else rng.randrange(c.n_entities)
        facts.append((src, rng.randrange(c.n_relations), rng.randrange(c.n_entities)))
    return facts


def request_fields(c: GraphCase) -> dict:
    """Fields of a GraphMemoryRequest (chunks as dicts of GraphRetentionChunk fields)."""
    rng = random.Random(c.seed)
    q_anchor = rng.randrange(c.n_entities)
    q_facts = _facts(rng, c.query_facts, q_anchor, c)
    q_rel = c.n_relations + 5 if c.unseen_query_relation else q_facts[0][1]
    chunks = []
    span = max(1, c.seq_len // (c.n_chunks + 2))
    for i in range(c.n_chunks):
        anchor = rng.randrange(c.n_entities)
        start = rng.randrange(0, max(1, c.seq_len - span))
        end = start + rng.randrange(span // 2, span + 1)
        chunks.append(dict(anchor=anchor, span=(start, end), facts=_facts(rng, c.chunk_facts, anchor, c),
                           shuffle_seed=(c.seed * 10 + i) if c.shuffle else None))
    return dict(query_anchor=q_anchor, query_relation=q_rel, query_facts=q_facts, chunks=chunks,
                normalize=c.normalize, shuffle_seed=(c.seed * 7) if c.shuffle else None)


def build_request(module, c: GraphCase):
    """A request of ``module``'s own classes (the reference's or this package's)."""
    f = request_fields(c)
    chunks = [module.GraphRetentionChunk(**ch) for ch in f.pop("chunks")]
    return module.GraphMemoryRequest(chunks=chunks, **f)


def build_model(module, c: GraphCase):
    cfg = module.GraphMemoryConfig(**c.geometry)
    model = module.GraphMemory17L(cfg)
    shapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    model.load_state_dict(seeded_state_dict(shapes, c.seed))
    return model.eval()


def cache_layers(c: GraphCase):
    """Seeded bf16 K/V layers for the cache part of a case."""
    _, B, H, D, L = c.cache
    g = torch.Generator().manual_seed(c.seed + 500)
    return [(torch.randn(B, H, c.seq_len, D, generator=g).to(torch.bfloat16),
             torch.randn(B, H, c.seq_len, D, generator=g).to(torch.bfloat16)) for _ in range(L)]
