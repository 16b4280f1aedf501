"""Layer-specific reference memory: data model, cache lifecycle and routing.

Semantics follow ``src/pra_torch/memory.py`` of the reference:

* entries become visible to routing only in ``READY`` state; ``begin_build`` /
  ``mark_failed`` / ``put`` / ``invalidate`` drive the lifecycle
  (``memory.py:235-241, 378-434``);
* routing is exact cosine search over L2-normalised gists (eps ``1e-12``),
  gist sets reduced by max / mean / logsumexp, chunk scores reduced to URI
  scores the same way (``memory.py:539-581``);
* ``hierarchical`` selects the top URIs, then the top chunks inside each; ties
  are ordered by ``(-score, uri)`` and ``(-score, chunk_id)``
  (``memory.py:641-760``); ``global_chunks`` ranks chunks globally under both
  limits (``memory.py:1043-1071``); ``reference_first`` scores cached URI gists
  first (``memory.py:1005-1041``);
* ``PRABatchedMemoryCache`` routes query row ``i`` only against row cache
  ``i`` and forbids URI-only lookup (``memory.py:1217-1309``).

What differs is the execution: the packed routing index is built once per
``(layer, device, dtype)`` and scoring plus top-k run as tensor programs with a
single device-to-host copy of the *selected* indices (or, through
``routing_plan``, no host copy at all for the fused device path).  The scalar
per-chunk path (``routing_backend='legacy'``) is kept as the oracle.
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod
from collections import defaultdict
from dataclasses import dataclass, field
from enum import Enum
from types import SimpleNamespace
from typing import TYPE_CHECKING

import torch
import torch.nn.functional as F

from .gists.common import NORM_EPS, reduce_scores, score_gist_set

if TYPE_CHECKING:
    from ..config import PRAConfig


# ---------------------------------------------------------------------------
# Data model
# ---------------------------------------------------------------------------

@dataclass
class LayerKV:
    """Projected K/V of one chunk at one layer, each ``[1, heads, tokens, head_dim]``."""

    k: torch.Tensor
    v: torch.Tensor


ChunkKV = LayerKV


def _as_rows(t: torch.Tensor | None) -> torch.Tensor | None:
    return t.unsqueeze(0) if t is not None and t.ndim == 1 else t


@dataclass
class ChunkRoutingGist:
    """``[G,D]`` content gists (and optional paired value / summary gists) of one chunk."""

    k: torch.Tensor
    v: torch.Tensor | None = None
    method: str = "mean"
    summary_k: torch.Tensor | None = None
    metadata: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        self.k, self.v, self.summary_k = _as_rows(self.k), _as_rows(self.v), _as_rows(self.summary_k)
        if self.k.ndim != 2:
            raise ValueError(f"Chunk routing keys must be [gists,model], got {self.k.shape}.")
        if self.v is not None and self.v.shape != self.k.shape:
            raise ValueError("Chunk routing value gists must match key-gist shape.")


@dataclass
class ReferenceRoutingGists:
    """``[G,D]`` URI-level gists of one entry at one layer."""

    k: torch.Tensor
    v: torch.Tensor | None = None
    mode: str = "mean"
    metadata: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        self.k, self.v = _as_rows(self.k), _as_rows(self.v)
        if self.k.ndim != 2:
            raise ValueError(f"Reference routing keys must be [gists,model], got {self.k.shape}.")
        if self.v is not None and self.v.shape != self.k.shape:
            raise ValueError("Reference routing value gists must match key-gist shape.")


@dataclass
class ReferenceChunkMemory:
    """Detail K/V and routing gists for one provenance-preserving span."""

    chunk_id: str
    source_uri: str
    token_start: int
    token_end: int
    token_kv: ChunkKV
    routing_gist: ChunkRoutingGist
    char_start: int | None = None
    char_end: int | None = None
    metadata: dict = field(default_factory=dict)

    @property
    def token_count(self) -> int:
        return int(self.token_kv.k.shape[2])


@dataclass
class LayerReferenceMemory:
    chunks: list[ReferenceChunkMemory] = field(default_factory=list)


@dataclass
class PRACacheEntry:
    """One resolved URI: per-layer chunk lists, optional URI gists, provenance."""

    uri: str
    text: str
    layer_memory: dict[int, LayerReferenceMemory] = field(default_factory=dict)
    reference_gists_by_layer: dict[int, ReferenceRoutingGists] = field(default_factory=dict)
    child_uris: list[str] = field(default_factory=list)
    metadata: dict = field(default_factory=dict)


@dataclass(frozen=True)
class SelectedChunk:
    """A routed chunk with its scores and ranks (trace record)."""

    entry: PRACacheEntry
    chunk: ReferenceChunkMemory
    reference_score: float
    chunk_score: float
    layer_id: int
    reference_rank: int
    rank_within_reference: int
    winning_gist_index: int | None = None
    winning_gist_score: float | None = None
    gist_count: int = 1
    winning_reference_gist_index: int | None = None
    winning_reference_gist_score: float | None = None
    reference_gist_count: int = 0
    metadata: dict = field(default_factory=dict)

    @property
    def reference_uri(self) -> str:
        return self.entry.uri

    @property
    def chunk_id(self) -> str:
        return self.chunk.chunk_id

    @property
    def source_uri(self) -> str:
        return self.chunk.source_uri

    @property
    def token_start(self) -> int:
        return self.chunk.token_start

    @property
    def token_end(self) -> int:
        return self.chunk.token_end

    @property
    def selected_token_count(self) -> int:
        return self.chunk.token_count

    def as_trace_dict(self) -> dict:
        keys = ("reference_uri", "reference_score", "chunk_id", "chunk_score", "layer_id", "token_start",
                "token_end", "selected_token_count", "reference_rank", "rank_within_reference",
                "winning_gist_index", "winning_gist_score", "gist_count", "winning_reference_gist_index",
                "winning_reference_gist_score", "reference_gist_count", "metadata")
        return {key: getattr(self, key) for key in keys}


@dataclass(frozen=True)
class _ChunkHit:
    entry: PRACacheEntry
    chunk: ReferenceChunkMemory
    score: float
    routing_source: str
    winning_gist_index: int | None
    winning_gist_score: float | None
    gist_count: int


@dataclass(frozen=True)
class _ReferenceHit:
    entry: PRACacheEntry
    score: float
    winning_gist_index: int | None
    winning_gist_score: float | None
    gist_count: int


class CacheBuildState(str, Enum):
    MISSING = "missing"
    BUILDING = "building"
    READY = "ready"
    FAILED = "failed"


def _aggregate(scores: list[float], mode: str) -> float:
    if not scores:
        return float("-inf")
    if mode == "max":
        return max(scores)
    if mode == "mean":
        return sum(scores) / len(scores)
    if mode == "logsumexp":
        top = max(scores)
        return top + math.log(sum(math.exp(s - top) for s in scores))
    raise ValueError(f"Unsupported reference score aggregation: {mode}")


# ---------------------------------------------------------------------------
# Packed routing index
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class RoutingIndex:
    """One layer's gists packed for exact batched search.

    ``gists`` ``[C,G,D]`` L2-normalised, ``gist_mask`` ``[C,G]``;
    ``ref_chunks`` ``[R,Cr]`` maps URI slots (sorted by URI) to chunk rows,
    ``ref_chunk_mask`` marks the valid slots.  ``chunk_id_rank`` is each chunk's
    position in lexical ``chunk_id`` order within its URI (ties on score are
    broken by it, so ``uri#chunk=10`` sorts before ``uri#chunk=2``).
    """

    records: tuple[tuple[PRACacheEntry, ReferenceChunkMemory], ...]
    gists: torch.Tensor
    gist_mask: torch.Tensor
    reference_entries: tuple[PRACacheEntry, ...]
    ref_chunks: torch.Tensor
    ref_chunk_mask: torch.Tensor
    ref_chunks_host: tuple[tuple[int, ...], ...]
    chunk_id_rank: tuple[int, ...]

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.gists, self.gist_mask, self.ref_chunks,
                                                           self.ref_chunk_mask))


def build_routing_index(entries: list[PRACacheEntry], layer_id: int, device, dtype) -> RoutingIndex | None:
    records = [(e, c) for e in entries if layer_id in e.layer_memory for c in e.layer_memory[layer_id].chunks]
    if not records:
        return None
    sets = [c.routing_gist.k.to(device, dtype) for _, c in records]
    counts = torch.tensor([int(s.shape[0]) for s in sets], device=device)
    width = int(counts.max())
    if width == 1:
        packed = torch.stack([s[0] for s in sets]).unsqueeze(1)
    else:
        packed = torch.zeros((len(sets), width, sets[0].shape[-1]), device=device, dtype=dtype)
        for row, s in enumerate(sets):
            packed[row, : s.shape[0]] = s
    mask = torch.arange(width, device=device)[None, :] < counts[:, None]
    packed = F.normalize(packed, dim=-1, eps=NORM_EPS)

    by_uri: dict[str, list[int]] = defaultdict(list)
    entry_of: dict[str, PRACacheEntry] = {}
    for row, (entry, _) in enumerate(records):
        by_uri[entry.uri].append(row)
        entry_of[entry.uri] = entry
    uris = sorted(by_uri)
    span = max(len(by_uri[u]) for u in uris)
    ref_chunks = torch.tensor([by_uri[u] + [0] * (span - len(by_uri[u])) for u in uris], dtype=torch.long,
                              device=device)
    ref_mask = torch.tensor([[True] * len(by_uri[u]) + [False] * (span - len(by_uri[u])) for u in uris],
                            dtype=torch.bool, device=device)
    rank = [0] * len(records)
    for u in uris:
        for position, row in enumerate(sorted(by_uri[u], key=lambda r: records[r][1].chunk_id)):
            rank[row] = position
    return RoutingIndex(tuple(records), packed, mask, tuple(entry_of[u] for u in uris), ref_chunks, ref_mask,
                        tuple(tuple(by_uri[u]) for u in uris), tuple(rank))


def score_index(query: torch.Tensor, index: RoutingIndex, aggregation: str):
    """``[B,D]`` queries -> (chunk score ``[B,C]``, winning gist ``[B,C]``, winning score ``[B,C]``)."""
    unit = F.normalize(query, dim=-1, eps=NORM_EPS)
    if index.gists.shape[1] == 1:
        scores = (unit @ index.gists[:, 0, :].T).unsqueeze(-1)
    else:
        scores = torch.einsum("bd,cgd->bcg", unit, index.gists)
    valid = index.gist_mask.unsqueeze(0).expand_as(scores)
    win_score, win_index = scores.masked_fill(~valid, float("-inf")).max(dim=-1)
    aggregate = win_score if aggregation == "max" else reduce_scores(scores, valid, aggregation)
    return aggregate, win_index, win_score


def reference_scores(chunk_scores: torch.Tensor, index: RoutingIndex, aggregation: str) -> torch.Tensor:
    grouped = chunk_scores[:, index.ref_chunks]
    valid = index.ref_chunk_mask.unsqueeze(0).expand_as(grouped)
    return reduce_scores(grouped, valid, aggregation)


@dataclass
class HierarchicalSelection:
    """Device tensors of one hierarchical routing decision (no host copy yet).

    ``ref_index`` / ``ref_score`` ``[B,k_ref]`` and ``chunk_index`` /
    ``chunk_score`` / ``win_index`` / ``win_score`` ``[B,k_ref,k_chunk]``;
    ``chunk_valid`` masks slots past a URI's chunk count.
    """

    ref_index: torch.Tensor
    ref_score: torch.Tensor
    chunk_index: torch.Tensor
    chunk_score: torch.Tensor
    win_index: torch.Tensor
    win_score: torch.Tensor
    chunk_valid: torch.Tensor


def hierarchical_select(index: RoutingIndex, chunk_scores, ref_scores, win_index, win_score, k_ref: int,
                        k_chunk: int) -> HierarchicalSelection | None:
    k_ref = min(int(k_ref), len(index.reference_entries))
    if k_ref == 0:
        return None
    top_ref_score, top_ref = torch.topk(ref_scores, k=k_ref, dim=-1, largest=True, sorted=True)
    grouped = chunk_scores[:, index.ref_chunks].masked_fill(~index.ref_chunk_mask.unsqueeze(0), float("-inf"))
    picked = torch.gather(grouped, 1, top_ref.unsqueeze(-1).expand(-1, -1, grouped.shape[-1]))
    k_chunk = min(int(k_chunk), int(index.ref_chunks.shape[1]))
    _, slots = torch.topk(picked, k=k_chunk, dim=-1, largest=True, sorted=True)
    rows = index.ref_chunks[top_ref]
    chunk = torch.gather(rows, 2, slots)
    flat = chunk.flatten(1)
    valid = torch.gather(index.ref_chunk_mask[top_ref], 2, slots)
    return HierarchicalSelection(
        top_ref, top_ref_score, chunk, torch.gather(chunk_scores, 1, flat).view_as(chunk),
        torch.gather(win_index, 1, flat).view_as(chunk), torch.gather(win_score, 1, flat).view_as(chunk), valid)


# ---------------------------------------------------------------------------
# Cache contract
# ---------------------------------------------------------------------------

class PRAMemoryCache(ABC):
    """Storage plus layer-aware, batch-isolated routing."""

    @abstractmethod
    def put(self, entry: PRACacheEntry) -> None: ...

    @abstractmethod
    def get(self, uri: str) -> PRACacheEntry | None: ...

    @abstractmethod
    def has(self, uri: str) -> bool: ...

    @abstractmethod
    def all_entries(self) -> list[PRACacheEntry]: ...

    @abstractmethod
    def clear(self) -> None: ...

    @abstractmethod
    def is_empty(self) -> bool: ...

    @abstractmethod
    def search(self, query: torch.Tensor, layer_id: int, config: "PRAConfig") -> list[list[SelectedChunk]]: ...

    @property
    def entries(self) -> dict[str, PRACacheEntry]:
        return {entry.uri: entry for entry in self.all_entries()}

    def __len__(self) -> int:
        return len(self.all_entries())


def _selected(hit: _ChunkHit, reference_score, layer_id, ref_rank, chunk_rank,
              reference_hit: _ReferenceHit | None = None) -> SelectedChunk:
    meta = hit.entry.metadata
    ref = reference_hit
    return SelectedChunk(
        entry=hit.entry, chunk=hit.chunk, reference_score=reference_score, chunk_score=hit.score,
        layer_id=layer_id, reference_rank=ref_rank, rank_within_reference=chunk_rank,
        winning_gist_index=hit.winning_gist_index, winning_gist_score=hit.winning_gist_score,
        gist_count=hit.gist_count, winning_reference_gist_index=ref.winning_gist_index if ref else None,
        winning_reference_gist_score=ref.winning_gist_score if ref else None,
        reference_gist_count=ref.gist_count if ref else 0,
        metadata={"routing_source": hit.routing_source, "reference_source": meta.get("source", "reference"),
                  "implicit_reference": bool(meta.get("implicit", False)),
                  "reference_display_name": meta.get("display_name", hit.entry.uri)})


# ---------------------------------------------------------------------------
# Scalar scoring (the oracle path) and the host-side strategies
# ---------------------------------------------------------------------------

def _augmented_gists(gist: ChunkRoutingGist, summary_k: torch.Tensor) -> torch.Tensor:
    """``augment`` summary mode: every content gist moved towards the mean summary direction."""
    boost = F.normalize(summary_k.mean(dim=0), dim=-1)
    return F.normalize(F.normalize(gist.k, dim=-1) + boost.unsqueeze(0), dim=-1)


def score_chunk(query: torch.Tensor, entry, chunk, config) -> _ChunkHit:
    """One chunk's cosine routing score for one ``[D]`` query (content gists, optionally combined
    with the chunk's summary gists as ``config.summary_mode`` says)."""
    gist, agg = chunk.routing_gist, config.gist_score_aggregation
    content = score_gist_set(query, gist.k, agg)
    score, source = content.aggregate_score, "content"
    if config.use_summary and gist.summary_k is not None:
        summary_k = _as_rows(gist.summary_k)
        mode = config.summary_mode
        if mode == "replace":
            score, source = score_gist_set(query, summary_k, agg).aggregate_score, "summary"
        elif mode == "hybrid":
            score, source = max(score, score_gist_set(query, summary_k, agg).aggregate_score), "hybrid"
        elif mode == "augment":
            score, source = score_gist_set(query, _augmented_gists(gist, summary_k), agg).aggregate_score, "augment"
        else:
            raise ValueError(f"Unsupported summary mode: {mode}")
    winner = content.winning_index
    win_score = None
    if content.per_gist_scores is not None and winner is not None:
        win_score = float(content.per_gist_scores[winner].cpu())
    return _ChunkHit(entry, chunk, score, source, winner, win_score, int(gist.k.shape[0]))


def _layer_chunks(entries, layer_id: int):
    return [(e, c) for e in entries if layer_id in e.layer_memory for c in e.layer_memory[layer_id].chunks]


def _by_reference(hits) -> dict[str, list[_ChunkHit]]:
    grouped: dict[str, list[_ChunkHit]] = defaultdict(list)
    for hit in hits:
        grouped[hit.entry.uri].append(hit)
    return grouped


def _chunk_order(hits):
    """Chunks best first; equal scores by chunk id (string order)."""
    return sorted(hits, key=lambda h: (-h.score, h.chunk.chunk_id))


def _reference_order(scores: dict[str, float]) -> list[str]:
    """URIs best first; equal scores by URI."""
    return sorted(scores, key=lambda u: (-scores[u], u))


def _reference_scores(grouped, aggregation: str) -> dict[str, float]:
    return {uri: _aggregate([h.score for h in hits], aggregation) for uri, hits in grouped.items()}


def _hierarchical(hits, layer_id, config) -> list[SelectedChunk]:
    """The top URIs by aggregated chunk score, then the top chunks inside each."""
    grouped = _by_reference(hits)
    scores = _reference_scores(grouped, config.reference_score_aggregation)
    picked = []
    for ref_rank, uri in enumerate(_reference_order(scores)[: config.top_k_references], start=1):
        best = _chunk_order(grouped[uri])[: config.top_k_chunks_per_reference]
        picked += [_selected(hit, scores[uri], layer_id, ref_rank, rank) for rank, hit in enumerate(best, start=1)]
    return picked


def _global_chunks(hits, layer_id, config) -> list[SelectedChunk]:
    """One global chunk ranking, admitting a chunk while both its URI's chunk quota and the URI quota allow."""
    scores = _reference_scores(_by_reference(hits), config.reference_score_aggregation)
    admitted: dict[str, int] = {}  # uri -> chunks taken, in admission order
    picked = []
    for hit in sorted(hits, key=lambda h: (-h.score, h.entry.uri, h.chunk.chunk_id)):
        uri = hit.entry.uri
        taken = admitted.get(uri)
        if taken is None:
            if len(admitted) >= config.top_k_references:
                continue
            taken = admitted[uri] = 0
        if taken >= config.top_k_chunks_per_reference:
            continue
        admitted[uri] = taken + 1
        picked.append(_selected(hit, scores[uri], layer_id, list(admitted).index(uri) + 1, taken + 1))
    return picked


_HOST_STRATEGIES = {"hierarchical": _hierarchical, "global_chunks": _global_chunks}


def _rankings(hits, config, *, reference_scores=None) -> list[dict]:
    """Every URI and chunk with its rank and score (routing metrics and rank diagnostics)."""
    grouped = _by_reference(hits)
    scores = reference_scores if reference_scores is not None else \
        _reference_scores(grouped, config.reference_score_aggregation)
    table = []
    for ref_rank, uri in enumerate(_reference_order(scores), start=1):
        chunks = [{"chunk_id": h.chunk.chunk_id, "chunk_rank": rank, "chunk_score": float(h.score),
                   "token_start": h.chunk.token_start, "token_end": h.chunk.token_end, "gist_count": h.gist_count,
                   "winning_gist_index": h.winning_gist_index, "winning_gist_score": h.winning_gist_score}
                  for rank, h in enumerate(_chunk_order(grouped.get(uri, [])), start=1)]
        table.append({"reference_uri": uri, "reference_rank": ref_rank, "reference_score": float(scores[uri]),
                      "chunks": chunks})
    return table


@dataclass
class _Slot:
    """One URI's lifecycle record: the state, the entry once ready, the failure once failed."""

    state: CacheBuildState
    entry: PRACacheEntry | None = None
    failure: str | None = None


class PRASimpleMemoryCache(PRAMemoryCache):
    """In-process cache: one lifecycle table, per-layer packed routing indexes, three strategies.

    Only ``READY`` URIs are visible (``get``, ``all_entries``, routing); any change of the
    table drops the packed indexes, which are rebuilt on the next search.
    """

    def __init__(self):
        self._slots: dict[str, _Slot] = {}
        self._last_rankings_by_layer: dict[int, list[list[dict]]] = {}
        self._indexes: dict[tuple, RoutingIndex] = {}
        self.resolution_events: list = []
        self.dependencies: list = []

    # -- lifecycle -----------------------------------------------------
    def invalidate_routing_indexes(self) -> None:
        self._indexes.clear()

    def _set(self, uri: str, slot: _Slot | None) -> None:
        if slot is None:
            self._slots.pop(uri, None)
        else:
            self._slots[uri] = slot
        self.invalidate_routing_indexes()

    def _ready(self):
        return ((uri, slot.entry) for uri, slot in self._slots.items() if slot.state is CacheBuildState.READY)

    @property
    def entries(self) -> dict[str, PRACacheEntry]:
        return dict(self._ready())

    def begin_build(self, uri: str) -> None:
        self._set(uri, _Slot(CacheBuildState.BUILDING))

    def mark_failed(self, uri: str, error: Exception | str) -> None:
        self._set(uri, _Slot(CacheBuildState.FAILED, failure=str(error)))

    def put(self, entry: PRACacheEntry) -> None:
        self._set(entry.uri, _Slot(CacheBuildState.READY, entry))

    def invalidate(self, uri: str) -> None:
        self._set(uri, None)

    def clear(self) -> None:
        self._slots.clear()
        self._last_rankings_by_layer.clear()
        self.invalidate_routing_indexes()

    def state(self, uri: str) -> CacheBuildState:
        slot = self._slots.get(uri)
        return CacheBuildState.MISSING if slot is None else slot.state

    def failure(self, uri: str) -> str | None:
        slot = self._slots.get(uri)
        return None if slot is None else slot.failure

    def get(self, uri: str) -> PRACacheEntry | None:
        slot = self._slots.get(uri)
        return slot.entry if slot is not None and slot.state is CacheBuildState.READY else None

    def has(self, uri: str) -> bool:
        return self.get(uri) is not None

    def all_entries(self) -> list[PRACacheEntry]:
        return [entry for _, entry in self._ready()]

    def is_empty(self) -> bool:
        return next(self._ready(), None) is None

    def layer_counts(self, layer_id: int) -> dict[str, int]:
        entries = [e for e in self.all_entries() if layer_id in e.layer_memory]
        chunks = [c for _, c in _layer_chunks(entries, layer_id)]
        ref_gists = [e.reference_gists_by_layer[layer_id] for e in entries if layer_id in e.reference_gists_by_layer]
        return {"references": len(entries), "chunks": len(chunks), "tokens": sum(c.token_count for c in chunks),
                "chunk_gists": sum(int(c.routing_gist.k.shape[0]) for c in chunks),
                "reference_gists": sum(int(g.k.shape[0]) for g in ref_gists)}

    def last_rankings(self, layer_id: int) -> list[list[dict]]:
        return self._last_rankings_by_layer.get(layer_id, [])

    # -- packed index --------------------------------------------------
    def routing_index(self, layer_id: int, query: torch.Tensor, *, reuse: bool = True) -> RoutingIndex | None:
        key = (int(layer_id), str(query.device), query.dtype)
        index = self._indexes.get(key) if reuse else None
        if index is None:
            index = build_routing_index(self.all_entries(), layer_id, query.device, query.dtype)
            if reuse and index is not None:
                self._indexes[key] = index
        return index

    def prepare_routing_index(self, layer_id: int, query: torch.Tensor, *, force_rebuild: bool = False) -> dict:
        """Build (or reuse) the packed index and report its size (warm-up / benchmarks)."""
        query = query.unsqueeze(0) if query.ndim == 1 else query
        key = (int(layer_id), str(query.device), query.dtype)
        reused = key in self._indexes and not force_rebuild
        if force_rebuild:
            self._indexes.pop(key, None)
        index = self.routing_index(layer_id, query, reuse=True)
        if index is None:
            return {"reused": reused, "candidate_chunks": 0, "candidate_gists": 0, "index_bytes": 0}
        return {"reused": reused, "candidate_chunks": len(index.records),
                "candidate_gists": int(index.gist_mask.sum().item()), "index_bytes": index.nbytes}

    # -- scoring ---------------------------------------------------------
    _score_chunk = staticmethod(score_chunk)

    def _score_chunks(self, query, layer_id, config, *, entries=None) -> list[list[_ChunkHit]]:
        records = _layer_chunks(self.all_entries() if entries is None else entries, layer_id)
        return [[score_chunk(row, e, c, config) for e, c in records] for row in query]

    def _tensor_hits(self, query, layer_id, config) -> tuple:
        index = self.routing_index(layer_id, query, reuse=config.cache_build_mode == "detached")
        if index is None:
            return [[] for _ in range(query.shape[0])], None, None
        scores = score_index(query, index, config.gist_score_aggregation)
        table = torch.stack((scores[0], scores[2], scores[1].to(scores[0].dtype)), dim=-1).detach().cpu()
        hits = [[_ChunkHit(e, c, float(row[i, 0]), "content", int(row[i, 2]), float(row[i, 1]),
                           int(c.routing_gist.k.shape[0])) for i, (e, c) in enumerate(index.records)]
                for row in table]
        return hits, index, scores

    @staticmethod
    def _fallback_reference_gists(entry: PRACacheEntry, layer_id: int, config):
        """URI gists derived from the chunk gists (``mean`` or ``last``) when none were built."""
        memory = entry.layer_memory.get(layer_id)
        if memory is None or not memory.chunks:
            return None
        mode = config.reference_level_gist_mode
        if mode is None:
            raise ValueError("search_strategy='reference_first' requires reference_level_gist_mode.")
        if mode not in {"mean", "last"}:
            raise RuntimeError(f"Reference gists for mode {mode!r} must be created during cache construction.")
        gists = [c.routing_gist for c in memory.chunks]
        keys = torch.cat([g.k for g in gists], dim=0)
        values = torch.cat([g.v for g in gists], dim=0) if all(g.v is not None for g in gists) else None
        pick = (lambda t: t.mean(dim=0, keepdim=True)) if mode == "mean" else (lambda t: t[-1:].clone())
        made = ReferenceRoutingGists(k=pick(keys), v=None if values is None else pick(values), mode=mode, metadata={
            "requested_gists": int(config.reference_gists_per_reference), "actual_gists": 1, "legacy_fallback": True})
        entry.reference_gists_by_layer[layer_id] = made
        return made

    def _score_references(self, query, layer_id, config) -> list[_ReferenceHit]:
        if config.reference_level_gist_mode is None:
            raise ValueError("search_strategy='reference_first' requires reference_level_gist_mode.")
        hits = []
        for entry in self.all_entries():
            gists = entry.reference_gists_by_layer.get(layer_id) or self._fallback_reference_gists(entry, layer_id,
                                                                                                   config)
            if gists is None:
                continue
            s = score_gist_set(query, gists.k, config.reference_gist_score_aggregation)
            win = None
            if s.per_gist_scores is not None and s.winning_index is not None:
                win = float(s.per_gist_scores[s.winning_index].cpu())
            hits.append(_ReferenceHit(entry, s.aggregate_score, s.winning_index, win, int(gists.k.shape[0])))
        return hits

    # -- strategies ------------------------------------------------------
    _serialize_rankings = staticmethod(_rankings)

    def _hierarchical_from_tensors(self, hits_by_row, index: RoutingIndex, scores, layer_id, config):
        chunk_scores, win_index, win_score = scores
        ref_scores = reference_scores(chunk_scores, index, config.reference_score_aggregation)
        sel = hierarchical_select(index, chunk_scores, ref_scores, win_index, win_score, config.top_k_references,
                                  config.top_k_chunks_per_reference)
        if sel is None:
            return [[] for _ in range(chunk_scores.shape[0])]
        ref_i, ref_s, chunk_i, chunk_s, win_i, win_s = (
            t.detach().cpu().tolist() for t in (sel.ref_index, sel.ref_score, sel.chunk_index, sel.chunk_score,
                                                sel.win_index, sel.win_score))
        k_chunk = sel.chunk_index.shape[-1]
        rows = []
        for b in range(len(ref_i)):
            refs = sorted(range(len(ref_i[b])), key=lambda j: (-ref_s[b][j], index.reference_entries[ref_i[b][j]].uri))
            row = []
            for ref_rank, j in enumerate(refs, start=1):
                n_valid = min(k_chunk, len(index.ref_chunks_host[ref_i[b][j]]))
                slots = sorted(range(n_valid),
                               key=lambda s: (-chunk_s[b][j][s], index.records[chunk_i[b][j][s]][1].chunk_id))
                for chunk_rank, slot in enumerate(slots, start=1):
                    c = chunk_i[b][j][slot]
                    entry, chunk = index.records[c]
                    hit = hits_by_row[b][c] if hits_by_row is not None else _ChunkHit(
                        entry, chunk, float(chunk_s[b][j][slot]), "content", int(win_i[b][j][slot]),
                        float(win_s[b][j][slot]), int(chunk.routing_gist.k.shape[0]))
                    row.append(_selected(hit, float(ref_s[b][j]), layer_id, ref_rank, chunk_rank))
            rows.append(row)
        return rows

    def _reference_first(self, query, layer_id, config) -> list[SelectedChunk]:
        """Score the URI gists first, then only the chunks of the best URIs."""
        ref_hits = sorted(self._score_references(query, layer_id, config),
                          key=lambda h: (-h.score, h.entry.uri))[: config.top_k_references]
        if not ref_hits:
            return []
        grouped = _by_reference(self._score_chunks(query.unsqueeze(0), layer_id, config,
                                                   entries=[h.entry for h in ref_hits])[0])
        picked = []
        for ref_rank, rh in enumerate(ref_hits, start=1):
            best = _chunk_order(grouped[rh.entry.uri])[: config.top_k_chunks_per_reference]
            picked += [_selected(h, rh.score, layer_id, ref_rank, r, rh) for r, h in enumerate(best, start=1)]
        return picked

    def search(self, query: torch.Tensor, layer_id: int, config: "PRAConfig") -> list[list[SelectedChunk]]:
        """Route ``[B,D]`` (or ``[D]``) queries with the configured strategy; rows never mix."""
        query = query.unsqueeze(0) if query.ndim == 1 else query
        if query.ndim != 2:
            raise ValueError(f"Expected query [batch,model] or [model], got {tuple(query.shape)}.")
        empty = [[] for _ in range(query.shape[0])]
        keep_rankings = bool(config.collect_routing_metrics or config.collect_rank_diagnostics)
        strategy = config.search_strategy
        rankings: list = empty
        if config.top_k_references == 0 or config.top_k_chunks_per_reference == 0:
            selected = empty
        elif strategy == "reference_first":
            selected, rankings = [], []
            for row in query:
                selected.append(self._reference_first(row, layer_id, config))
                refs = {h.entry.uri: h.score for h in self._score_references(row, layer_id, config)} \
                    if keep_rankings else None
                rankings.append(_rankings(self._score_chunks(row.unsqueeze(0), layer_id, config)[0], config,
                                          reference_scores=refs) if keep_rankings else [])
        elif config.routing_backend == "tensorized" and not config.use_summary and strategy == "hierarchical":
            if keep_rankings:  # rankings need every chunk's score on the host
                hits_by_row, index, scores = self._tensor_hits(query, layer_id, config)
                if index is not None:
                    rankings = [_rankings(h, config) for h in hits_by_row]
            else:
                index = self.routing_index(layer_id, query, reuse=config.cache_build_mode == "detached")
                hits_by_row, scores = None, None if index is None else score_index(
                    query, index, config.gist_score_aggregation)
            selected = empty if index is None else \
                self._hierarchical_from_tensors(hits_by_row, index, scores, layer_id, config)
        else:
            if config.routing_backend == "tensorized" and not config.use_summary:
                hits_by_row = self._tensor_hits(query, layer_id, config)[0]
            else:
                hits_by_row = self._score_chunks(query, layer_id, config)
            choose = _HOST_STRATEGIES.get(strategy)
            if choose is None:
                raise ValueError(f"Unsupported search_strategy: {strategy}")
            selected = [choose(hits, layer_id, config) for hits in hits_by_row]
            rankings = [_rankings(hits, config) if keep_rankings else [] for hits in hits_by_row]
        self._last_rankings_by_layer[layer_id] = rankings
        return selected

    def search_by_routing_key(self, query: torch.Tensor, layer_id: int, top_k: int = 2):
        """Legacy one-chunk-per-URI lookup returning ``(entry, reference_score)`` pairs."""
        settings = SimpleNamespace(
            top_k_references=top_k, top_k_chunks_per_reference=1, search_strategy="hierarchical",
            routing_backend="tensorized", reference_score_aggregation="max", reference_level_gist_mode=None,
            reference_gists_per_reference=1, reference_gist_score_aggregation="max", gist_score_aggregation="max",
            use_summary=False, summary_mode="replace", cache_build_mode="detached", collect_routing_metrics=False,
            collect_rank_diagnostics=False)
        return [[(hit.entry, hit.reference_score) for hit in row] for row in self.search(query, layer_id, settings)]


class PRABatchedMemoryCache(PRAMemoryCache):
    """Row-local namespaces for one batched forward: query row ``i`` sees only ``row_caches[i]``."""

    def __init__(self, row_caches: list[PRAMemoryCache]):
        self.row_caches = list(row_caches)

    @property
    def entries(self) -> dict[str, PRACacheEntry]:
        raise RuntimeError("PRABatchedMemoryCache has no flat entries view; inspect row_caches explicitly.")

    def put(self, entry: PRACacheEntry) -> None:
        raise RuntimeError("Cannot put entries directly into PRABatchedMemoryCache.")

    def get(self, uri: str) -> PRACacheEntry | None:
        raise RuntimeError("Batched cache lookup requires an explicit row cache.")

    def has(self, uri: str) -> bool:
        raise RuntimeError("Batched cache membership requires an explicit row cache.")

    def all_entries(self) -> list[PRACacheEntry]:
        return [entry for cache in self.row_caches for entry in cache.all_entries()]

    def clear(self) -> None:
        for cache in self.row_caches:
            cache.clear()

    def invalidate_routing_indexes(self) -> None:
        for cache in self.row_caches:
            if hasattr(cache, "invalidate_routing_indexes"):
                cache.invalidate_routing_indexes()

    def is_empty(self) -> bool:
        return all(cache.is_empty() for cache in self.row_caches)

    def search(self, query: torch.Tensor, layer_id: int, config) -> list[list[SelectedChunk]]:
        query = query.unsqueeze(0) if query.ndim == 1 else query
        if query.ndim != 2:
            raise ValueError(f"Expected query [batch,model], got {tuple(query.shape)}.")
        if query.shape[0] != len(self.row_caches):
            raise ValueError("Routing-query batch size must match row-local cache count: "
                             f"{query.shape[0]} != {len(self.row_caches)}.")
        return [cache.search(query[i:i + 1], layer_id, config)[0] for i, cache in enumerate(self.row_caches)]

    def last_rankings(self, layer_id: int) -> list[list[dict]]:
        out = []
        for cache in self.row_caches:
            rows = cache.last_rankings(layer_id) if hasattr(cache, "last_rankings") else []
            out.append(rows[0] if rows else [])
        return out

    def __len__(self) -> int:
        return sum(len(cache) for cache in self.row_caches)
