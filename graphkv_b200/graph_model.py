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

def _slot(mapping: dict[int, int], key: int, limit: int) -> int:
    """Local id of a global id: first-seen order, saturating at ``limit - 1``
    (``graph_model.py:425-428``)."""
    if key not in mapping:
        mapping[key] = min(len(mapping), limit - 1)
    return mapping[key]


def build_fact_bank(anchor: int, facts: Iterable[Fact], *, num_facts: int, num_entities: int, num_relations: int,
                    shuffle_seed: int | None = None) -> GraphFactBank:
    """Relabel a fact list into local slots, anchor entity = slot 0, keep the
    first ``num_facts`` facts, zero-pad (``graph_model.py:362-388``).  The
    optional shuffle is Python's ``random.Random(seed).shuffle``."""
    items = list(facts)
    if shuffle_seed is not None:
        random.Random(shuffle_seed).shuffle(items)
    entities: dict[int, int] = {int(anchor): 0}
    relations: dict[int, int] = {}
    for s, r, d in items:
        _slot(entities, int(s), num_entities)
        _slot(entities, int(d), num_entities)
        _slot(relations, int(r), num_relations)
    kept = items[:num_facts]
    table = torch.zeros(3, num_facts, dtype=torch.long)
    if kept:
        table[:, : len(kept)] = torch.tensor(
            [[entities.get(int(s), 0), relations.get(int(r), 0), entities.get(int(d), 0)] for s, r, d in kept],
            dtype=torch.long).t()
    return GraphFactBank(src=table[0].clone(), rel=table[1].clone(), dst=table[2].clone(),
                         relation_map=relations, entity_map=entities)


def build_query_bank(anchor: int, query_relation: int, facts: Iterable[Fact], cfg: GraphMemoryConfig,
                     shuffle_seed: int | None = None) -> GraphQueryBank:
    """Query facts; an unseen query relation maps to the last relation slot (``graph_model.py:391-406``)."""
    bank = build_fact_bank(anchor, facts, num_facts=cfg.num_facts, num_entities=cfg.num_entities,
                           num_relations=cfg.num_relations, shuffle_seed=shuffle_seed)
    return GraphQueryBank(facts=bank, query_relation=bank.relation_map.get(int(query_relation), cfg.num_relations - 1))


def build_candidate_bank(anchor: int, facts: Iterable[Fact], cfg: GraphMemoryConfig,
                         shuffle_seed: int | None = None) -> GraphFactBank:
    return build_fact_bank(anchor, facts, num_facts=cfg.num_cand_facts, num_entities=cfg.num_entities,
                           num_relations=cfg.num_relations, shuffle_seed=shuffle_seed)


def normalize_graph_scores(scores: torch.Tensor, *, mode: Normalize = "minmax") -> torch.Tensor:
    """Rank-preserving normalisation (``graph_model.py:337-359``): minmax maps to
    [0, 1] (all ones when the range is below 1e-8); zscore uses the population
    std (all zeros when it is below 1e-8)."""
    scores = scores.to(dtype=torch.float32)
    if mode == "none" or scores.numel() == 0:
        return scores
    if mode == "minmax":
        lo, hi = scores.min(), scores.max()
        if bool((hi - lo).abs() < 1.0e-8):
            return torch.ones_like(scores)
        return (scores - lo) / (hi - lo)
    if mode == "zscore":
        mean, std = scores.mean(), scores.std(unbiased=False)
        if bool(std < 1.0e-8):
            return torch.zeros_like(scores)
        return (scores - mean) / std
    raise ValueError("mode must be 'none', 'minmax', or 'zscore'.")


def _resolve_graph_device(device: str | torch.device) -> torch.device:
    if str(device) == "auto":
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")
    return torch.device(device)


def graph_mneme_chunk_scores(query: GraphQueryBank, candidates: Sequence[GraphFactBank], *,
                             model: GraphMemory17L | None = None, device: torch.device | str | None = None,
                             normalize: Normalize = "minmax") -> torch.Tensor:
    """Normalised scores of the candidate chunks (``graph_model.py:227-242``)."""
    if model is None:
        model = load_bundled_graph_model(device=device or "auto")
    target = _resolve_graph_device(device) if device is not None else next(model.parameters()).device
    model = model.to(target)
    return normalize_graph_scores(model.score(query, candidates, device=target), mode=normalize)


def graph_mneme_token_scores(seq_len: int, chunk_spans: Iterable[tuple[int, int]], query: GraphQueryBank,
                             candidates: Sequence[GraphFactBank], *, model: GraphMemory17L | None = None,
                             device: torch.device | str | None = None,
                             normalize: Normalize = "minmax") -> torch.Tensor:
    """One score per token: the max over the chunks covering it, 0 elsewhere (``graph_model.py:245-266``)."""
    from .core import chunk_scores_to_token_scores

    scores = graph_mneme_chunk_scores(query, candidates, model=model, device=device, normalize=normalize)
    return chunk_scores_to_token_scores(seq_len, chunk_spans, scores, device=scores.device)


def build_graph_mneme_token_scores(seq_len: int, *, query_anchor: int, query_relation: int,
                                   query_facts: Iterable[Fact], chunks: Sequence[GraphRetentionChunk],
                                   model: GraphMemory17L | None = None, device: torch.device | str | None = None,
                                   normalize: Normalize = "minmax", shuffle_seed: int | None = None) -> torch.Tensor:
    """Banks from the raw facts, chunk scores, token scores (``graph_model.py:269-312``)."""
    if model is None:
        model = load_bundled_graph_model(device=device or "auto")
    if device is not None:
        device = _resolve_graph_device(device)
    cfg = model.cfg
    query = build_query_bank(query_anchor, query_relation, query_facts, cfg, shuffle_seed=shuffle_seed)
    candidates = [build_candidate_bank(c.anchor, c.facts, cfg, shuffle_seed=c.shuffle_seed) for c in chunks]
    return graph_mneme_token_scores(seq_len, [c.span for c in chunks], query, candidates, model=model, device=device,
                                    normalize=normalize)


def graph_mneme_request_token_scores(seq_len: int, request: GraphMemoryRequest, *,
                                     model: GraphMemory17L | None = None,
                                     device: torch.device | str | None = None) -> torch.Tensor:
    """Score a ``GraphMemoryRequest`` over a cache of ``seq_len`` tokens (``graph_model.py:315-334``)."""
    return build_graph_mneme_token_scores(
        seq_len, query_anchor=request.query_anchor, query_relation=request.query_relation,
        query_facts=request.query_facts, chunks=request.chunks, model=model, device=device,
        normalize=request.normalize, shuffle_seed=request.shuffle_seed)
