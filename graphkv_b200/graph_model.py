"""Graph Mneme importance scores for ``quantize_hf_cache(graph_memory=...)``.

A ``GraphMemoryRequest`` (a query over a small knowledge graph plus candidate
text chunks, each backed by local facts) is scored by the Graph Mneme
transformer into one score per chunk; the chunk scores are normalised and
spread over the token positions of their spans, and the result drives the
same tier selection as explicit ``importance_scores``
(reference: ``src/graphkv/graph_model.py``, ``src/graphkv/core.py:775-797``).

The scorer runs as plain PyTorch on the device the cache lives on (it is a
6-layer, 256-wide encoder over at most 66 positions: a few milliseconds of
library GEMMs, off the compression path).  Its parameter names equal the
reference's so that a checkpoint trained for the reference loads unchanged;
the bundled weights are not part of this package, so
``load_bundled_graph_model`` looks for a ``latest.safetensors`` the user puts
in ``graphkv_b200/models/mneme-graph-17l/`` (or names with
``GRAPHKV_MNEME_WEIGHTS``) and raises ``FileNotFoundError`` otherwise.
"""
from __future__ import annotations

import os
import random
from dataclasses import dataclass, fields
from pathlib import Path
from typing import Iterable, Literal, Sequence

import torch
from torch import nn
from torch.nn import functional as F

Normalize = Literal["none", "minmax", "zscore"]
Fact = tuple[int, int, int]


@dataclass(frozen=True)
class GraphMemoryConfig:
    """Scorer geometry (reference ``graph_model.py:15-32``)."""

    model_name: str = "mneme-graph-17l"
    num_entities: int = 128
    num_facts: int = 64
    num_cand_facts: int = 32
    num_candidates: int = 64
    num_relations: int = 512
    d_model: int = 256
    num_heads: int = 8
    encoder_layers: int = 6
    dropout: float = 0.05
    num_global_relations: int = 0

    @classmethod
    def from_mapping(cls, data: dict) -> "GraphMemoryConfig":
        names = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in data.items() if k in names})


@dataclass(frozen=True)
class GraphFactBank:
    """Up to ``num_facts`` (src, rel, dst) facts in local slot ids (``graph_model.py:35-48``)."""

    src: torch.Tensor
    rel: torch.Tensor
    dst: torch.Tensor
    relation_map: dict[int, int]
    entity_map: dict[int, int]

    def as_batch(self, device: torch.device | str) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        return tuple(t.unsqueeze(0).to(device) for t in (self.src, self.rel, self.dst))


@dataclass(frozen=True)
class GraphQueryBank:
    facts: GraphFactBank
    query_relation: int


@dataclass(frozen=True)
class GraphRetentionChunk:
    """A token span ``[span[0], span[1])`` backed by local graph facts (``graph_model.py:57-64``)."""

    anchor: int
    span: tuple[int, int]
    facts: Sequence[Fact]
    shuffle_seed: int | None = None


@dataclass(frozen=True)
class GraphMemoryRequest:
    """Graph query plus candidate chunks for automatic KV-retention scoring (``graph_model.py:67-76``)."""

    query_anchor: int
    query_relation: int
    query_facts: Sequence[Fact]
    chunks: Sequence[GraphRetentionChunk]
    normalize: Normalize = "minmax"
    shuffle_seed: int | None = None


GraphMnemeRequest = GraphMemoryRequest


class FactGraphAttention(nn.Module):
    """Pre-norm encoder block: x += attn(LN(x)); x += FFN(LN(x)) (``graph_model.py:82-106``)."""

    def __init__(self, d_model: int, num_heads: int, dropout: float = 0.05):
        super().__init__()
        self.num_heads = num_heads
        self.norm = nn.LayerNorm(d_model, eps=1e-5)
        self.attn_in = nn.Linear(d_model, 3 * d_model)
        self.attn_out = nn.Linear(d_model, d_model)
        self.ff_norm = nn.LayerNorm(d_model, eps=1e-5)
        self.ff1 = nn.Linear(d_model, 4 * d_model)
        self.ff2 = nn.Linear(4 * d_model, d_model)
        self.drop = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, n, d = x.shape
        heads = self.attn_in(self.norm(x)).view(b, n, 3, self.num_heads, d // self.num_heads)
        q, k, v = heads.permute(2, 0, 3, 1, 4).unbind(0)  # each [b, heads, n, head_dim]
        mixed = F.scaled_dot_product_attention(q, k, v, dropout_p=0.0)
        x = x + self.drop(self.attn_out(mixed.transpose(1, 2).reshape(b, n, d)))
        return x + self.drop(self.ff2(F.gelu(self.ff1(self.ff_norm(x)))))


class GraphMemory17L(nn.Module):
    """Graph Mneme scorer (``graph_model.py:109-201``).

    Facts are embedded as MLP([E(src)+role_src, R(rel), E(dst)+role_dst]) plus a
    position; the query sequence is [query CLS, relation prototype, facts], a
    candidate sequence is [entity CLS, facts]; both run through the same
    encoder stack, and the score is <query vec, candidate vec> / temperature.
    """

    def __init__(self, cfg: GraphMemoryConfig):
        super().__init__()
        self.cfg = cfg
        d = cfg.d_model
        self.entity_emb = nn.Embedding(cfg.num_entities, d)
        self.rel_emb = nn.Embedding(cfg.num_relations, d)
        self.src_role = nn.Parameter(torch.zeros(d))
        self.dst_role = nn.Parameter(torch.zeros(d))
        self.fact_mlp = nn.Sequential(nn.Linear(3 * d, 3 * d), nn.GELU(), nn.Dropout(cfg.dropout), nn.Linear(3 * d, d))
        self.fact_pos = nn.Parameter(torch.zeros(1, max(cfg.num_facts, cfg.num_cand_facts), d))
        self.layers = nn.ModuleList(FactGraphAttention(d, cfg.num_heads, cfg.dropout) for _ in range(cfg.encoder_layers))
        self.query_cls = nn.Parameter(torch.zeros(1, 1, d))
        self.query_rel_proj = nn.Linear(d, d, bias=False)
        self.query_norm = nn.LayerNorm(d, eps=1e-5)
        self.query_head = nn.Linear(d, d, bias=False)
        self.entity_cls = nn.Parameter(torch.zeros(1, 1, d))
        self.entity_norm = nn.LayerNorm(d, eps=1e-5)
        self.entity_head = nn.Linear(d, d, bias=False)
        self.log_temp = nn.Parameter(torch.zeros(1))

    def _facts(self, src: torch.Tensor, rel: torch.Tensor, dst: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(fact content, content + position) for fact id tensors [batch, n_facts]."""
        triple = torch.cat([self.entity_emb(src) + self.src_role, self.rel_emb(rel),
                            self.entity_emb(dst) + self.dst_role], dim=-1)
        content = self.fact_mlp(triple)
        return content, content + self.fact_pos[:, : src.shape[1]]

    def _encode(self, seq: torch.Tensor) -> torch.Tensor:
        for block in self.layers:
            seq = block(seq)
        return seq[:, 0]

    def encode_query(self, fact_src: torch.Tensor, fact_rel: torch.Tensor, fact_dst: torch.Tensor,
                     query_relation: torch.Tensor) -> torch.Tensor:
        content, facts = self._facts(fact_src, fact_rel, fact_dst)
        # mean fact content over the facts that carry the query relation (0 when none do)
        hit = (fact_rel == query_relation.unsqueeze(1)).float()
        proto = (content * hit.unsqueeze(-1)).sum(1) / hit.sum(1, keepdim=True).clamp(min=1)
        cls = self.query_cls.expand(facts.shape[0], -1, -1)
        seq = torch.cat([cls, self.query_rel_proj(proto).unsqueeze(1), facts], dim=1)
        return self.query_head(self.query_norm(self._encode(seq)))

    def encode_entity(self, fact_src: torch.Tensor, fact_rel: torch.Tensor, fact_dst: torch.Tensor) -> torch.Tensor:
        _, facts = self._facts(fact_src, fact_rel, fact_dst)
        seq = torch.cat([self.entity_cls.expand(facts.shape[0], -1, -1), facts], dim=1)
        return self.entity_head(self.entity_norm(self._encode(seq)))

    @torch.no_grad()
    def score(self, query: GraphQueryBank, candidates: Sequence[GraphFactBank],
              device: torch.device | str | None = None) -> torch.Tensor:
        """One fp32 score per candidate, all candidates in one encoder batch."""
        if device is None:
            device = next(self.parameters()).device
        if len(candidates) == 0:
            return torch.empty(0, dtype=torch.float32, device=device)
        qvec = self.encode_query(*query.facts.as_batch(device),
                                 torch.tensor([query.query_relation], dtype=torch.long, device=device))
        ids = [torch.stack([getattr(c, f) for c in candidates]).to(device) for f in ("src", "rel", "dst")]
        cvecs = self.encode_entity(*ids)
        temp = self.log_temp.exp().clamp(0.1, 10.0)
        return (qvec @ cvecs.t()).squeeze(0) / temp


# ---------------------------------------------------------------------------
# weights
# ---------------------------------------------------------------------------

def bundled_graph_model_dir() -> Path:
    return Path(__file__).resolve().parent / "models" / "mneme-graph-17l"


def bundled_graph_model_metadata() -> dict[str, object]:
    """The scorer geometry the bundled checkpoint name stands for."""
    return {f.name: getattr(GraphMemoryConfig(), f.name) for f in fields(GraphMemoryConfig)}


def _weights_path() -> Path:
    env = os.environ.get("GRAPHKV_MNEME_WEIGHTS")
    return Path(env) if env else bundled_graph_model_dir() / "latest.safetensors"


def load_bundled_graph_model(device: str | torch.device = "auto") -> GraphMemory17L:
    """Load the Graph Mneme checkpoint (``graph_model.py:215-224``).  The weights
    are user-supplied: a missing file raises ``FileNotFoundError``, as the
    reference does when its weights are absent."""
    path = _weights_path()
    if not path.is_file():
        raise FileNotFoundError(
            f"Graph Mneme weights not found at {path}; place latest.safetensors there, set "
            "GRAPHKV_MNEME_WEIGHTS, or pass graph_mneme_model=GraphMemory17L(...) explicitly.")
    from safetensors.torch import load_file

    dev = _resolve_graph_device(device)
    model = GraphMemory17L(GraphMemoryConfig.from_mapping(bundled_graph_model_metadata())).to(dev)
    model.load_state_dict(load_file(str(path), device=str(dev)))
    return model.eval()


# ---------------------------------------------------------------------------
# requests -> fact banks -> scores
# ---------------------------------------------------------------------------

class _LocalIds:
    """First-seen numbering of global ids into ``limit`` local slots: the k-th
    new id gets slot k, and ids beyond the last slot share it
    (``graph_model.py:425-428``).  ``first`` takes slot 0."""

    def __init__(self, limit: int, first: int | None = None):
        self.limit = limit
        self.ids: dict[int, int] = {} if first is None else {int(first): 0}

    def add(self, key) -> None:
        self.ids.setdefault(int(key), min(len(self.ids), self.limit - 1))

    def __getitem__(self, key) -> int:
        return self.ids.get(int(key), 0)


def build_fact_bank(anchor: int, facts: Iterable[Fact], *, num_facts: int, num_entities: int, num_relations: int,
                    shuffle_seed: int | None = None) -> GraphFactBank:
    """A fact list in local ids (``graph_model.py:362-388``): entities numbered
    from the anchor (slot 0) in order of appearance, relations likewise, the
    first ``num_facts`` facts as (src, rel, dst) columns, zero-padded.  The
    optional shuffle is Python's ``random.Random(seed).shuffle``."""
    items = list(facts)
    if shuffle_seed is not None:
        random.Random(shuffle_seed).shuffle(items)
    entities, relations = _LocalIds(num_entities, first=anchor), _LocalIds(num_relations)
    for src, rel, dst in items:
        entities.add(src)
        entities.add(dst)
        relations.add(rel)
    table = torch.zeros(num_facts, 3, dtype=torch.long)
    local = [(entities[src], relations[rel], entities[dst]) for src, rel, dst in items[:num_facts]]
    if local:
        table[: len(local)] = torch.tensor(local, dtype=torch.long)
    return GraphFactBank(src=table[:, 0].contiguous(), rel=table[:, 1].contiguous(), dst=table[:, 2].contiguous(),
                         relation_map=relations.ids, entity_map=entities.ids)


def build_query_bank(anchor: int, query_relation: int, facts: Iterable[Fact], cfg: GraphMemoryConfig,
                     shuffle_seed: int | None = None) -> GraphQueryBank:
    """The query's fact bank; a query relation that none of its facts uses gets
    the last relation slot (``graph_model.py:391-406``)."""
    bank = build_fact_bank(anchor, facts, num_facts=cfg.num_facts, num_entities=cfg.num_entities,
                           num_relations=cfg.num_relations, shuffle_seed=shuffle_seed)
    rel = bank.relation_map.get(int(query_relation), cfg.num_relations - 1)
    return GraphQueryBank(facts=bank, query_relation=rel)


def build_candidate_bank(anchor: int, facts: Iterable[Fact], cfg: GraphMemoryConfig,
                         shuffle_seed: int | None = None) -> GraphFactBank:
    """A candidate chunk's fact bank (``num_cand_facts`` rows)."""
    return build_fact_bank(anchor, facts, num_facts=cfg.num_cand_facts, num_entities=cfg.num_entities,
                           num_relations=cfg.num_relations, shuffle_seed=shuffle_seed)


def _minmax(scores: torch.Tensor) -> torch.Tensor:
    lo, hi = scores.min(), scores.max()
    span = hi - lo
    return torch.ones_like(scores) if bool(span.abs() < 1.0e-8) else (scores - lo) / span


def _zscore(scores: torch.Tensor) -> torch.Tensor:
    centre, spread = scores.mean(), scores.std(unbiased=False)
    return torch.zeros_like(scores) if bool(spread < 1.0e-8) else (scores - centre) / spread


_NORMALIZERS = {"minmax": _minmax, "zscore": _zscore}


def normalize_graph_scores(scores: torch.Tensor, *, mode: Normalize = "minmax") -> torch.Tensor:
    """Rank-preserving rescaling of fp32 scores (``graph_model.py:337-359``):
    ``minmax`` onto [0, 1] (all ones for a range below 1e-8), ``zscore`` by the
    population standard deviation (all zeros below 1e-8), ``none`` unchanged."""
    scores = scores.to(dtype=torch.float32)
    if mode == "none" or scores.numel() == 0:
        return scores
    rescale = _NORMALIZERS.get(mode)
    if rescale is None:
        raise ValueError("mode must be 'none', 'minmax', or 'zscore'.")
    return rescale(scores)


def _resolve_graph_device(device: str | torch.device) -> torch.device:
    if str(device) == "auto":
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")
    return torch.device(device)


def _scoring_model(model: GraphMemory17L | None, device) -> tuple[GraphMemory17L, torch.device]:
    """The model that scores (the bundled one when none is given) moved to the
    requested device, or left on its own device when none is requested."""
    if model is None:
        model = load_bundled_graph_model(device=device or "auto")
    target = _resolve_graph_device(device) if device is not None else next(model.parameters()).device
    return model.to(target), target


def graph_mneme_chunk_scores(query: GraphQueryBank, candidates: Sequence[GraphFactBank], *,
                             model: GraphMemory17L | None = None, device: torch.device | str | None = None,
                             normalize: Normalize = "minmax") -> torch.Tensor:
    """Normalised relevance of each candidate chunk to the query (``graph_model.py:227-242``)."""
    model, target = _scoring_model(model, device)
    return normalize_graph_scores(model.score(query, candidates, device=target), mode=normalize)


def graph_mneme_token_scores(seq_len: int, chunk_spans: Iterable[tuple[int, int]], query: GraphQueryBank,
                             candidates: Sequence[GraphFactBank], *, model: GraphMemory17L | None = None,
                             device: torch.device | str | None = None,
                             normalize: Normalize = "minmax") -> torch.Tensor:
    """Chunk scores spread over token positions: each token takes the largest
    score of the chunks covering it, uncovered tokens 0 (``graph_model.py:245-266``)."""
    from .core import chunk_scores_to_token_scores

    per_chunk = graph_mneme_chunk_scores(query, candidates, model=model, device=device, normalize=normalize)
    return chunk_scores_to_token_scores(seq_len, chunk_spans, per_chunk, device=per_chunk.device)


def build_graph_mneme_token_scores(seq_len: int, *, query_anchor: int, query_relation: int,
                                   query_facts: Iterable[Fact], chunks: Sequence[GraphRetentionChunk],
                                   model: GraphMemory17L | None = None, device: torch.device | str | None = None,
                                   normalize: Normalize = "minmax", shuffle_seed: int | None = None) -> torch.Tensor:
    """Token scores from raw facts: the query and candidate banks are built with
    the model's sizes, then scored (``graph_model.py:269-312``)."""
    if model is None:
        model = load_bundled_graph_model(device=device or "auto")
    query = build_query_bank(query_anchor, query_relation, query_facts, model.cfg, shuffle_seed=shuffle_seed)
    banks = [build_candidate_bank(c.anchor, c.facts, model.cfg, shuffle_seed=c.shuffle_seed) for c in chunks]
    target = None if device is None else _resolve_graph_device(device)
    return graph_mneme_token_scores(seq_len, [c.span for c in chunks], query, banks, model=model, device=target,
                                    normalize=normalize)


_REQUEST_FIELDS = ("query_anchor", "query_relation", "query_facts", "chunks", "normalize", "shuffle_seed")


def graph_mneme_request_token_scores(seq_len: int, request: GraphMemoryRequest, *,
                                     model: GraphMemory17L | None = None,
                                     device: torch.device | str | None = None) -> torch.Tensor:
    """Token scores of a ``GraphMemoryRequest`` for a cache of ``seq_len`` tokens
    (``graph_model.py:315-334``)."""
    fields = {name: getattr(request, name) for name in _REQUEST_FIELDS}
    return build_graph_mneme_token_scores(seq_len, model=model, device=device, **fields)
