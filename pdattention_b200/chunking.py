"""Token-exact, provenance-preserving partitioning of reference sources.

Behaviour follows ``src/pra_torch/chunking.py`` of the reference:

* modes ``none`` / ``fixed`` (token windows, optional overlap) / ``markers``
  (literal markers or Markdown headings, with a token-exact fallback to fixed
  windows) / ``semantic`` (explicit plugin) (``chunking.py:315-432``);
* chunk identities are ``f"{uri}#chunk={i}"`` (``chunking.py:149-151``) -- note
  that this makes lexical and numeric order differ for ``i >= 10``, which the
  routing tie-break reproduces;
* oversized chunks are split at ``max_chunk_tokens`` and renumbered
  (``chunking.py:243-267``);
* a chunk cap applies ``truncate`` / ``merge_tail`` / ``error``
  (``chunking.py:180-212``).

The page table of the device memory store is built from the spans produced
here, so every span is an exact ``[token_start, token_end)`` slice of the
source token ids.
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field, replace
from typing import Protocol

CHUNK_MODES = ("none", "fixed", "markers", "semantic")


@dataclass(frozen=True)
class ChunkingConfig:
    """One partition policy, used both for encoding blocks and routing chunks."""

    mode: str = "fixed"
    chunk_tokens: int | None = None
    overlap_fraction: float = 0.0
    overlap_tokens: int = 0
    markers: tuple[str, ...] = ("<PRA_CHUNK>",)
    semantic_chunker: object | None = None

    def __post_init__(self) -> None:
        if self.mode not in CHUNK_MODES:
            raise ValueError(f"Unsupported chunking mode: {self.mode}")
        if self.chunk_tokens is not None and int(self.chunk_tokens) <= 0:
            raise ValueError("chunk_tokens must be positive or None.")
        if int(self.overlap_tokens) < 0:
            raise ValueError("overlap_tokens must be non-negative.")
        if not 0.0 <= float(self.overlap_fraction) < 1.0:
            raise ValueError("overlap_fraction must satisfy 0 <= value < 1.")
        if self.overlap_tokens and self.overlap_fraction:
            raise ValueError("Configure overlap_tokens or overlap_fraction, not both.")
        if self.mode == "semantic" and self.semantic_chunker is None:
            raise NotImplementedError("mode='semantic' requires an explicit semantic_chunker implementation.")

    @classmethod
    def from_value(cls, value) -> "ChunkingConfig":
        if isinstance(value, cls):
            return value
        if isinstance(value, dict):
            payload = dict(value)
            if "markers" in payload:
                payload["markers"] = tuple(payload["markers"] or ())
            return cls(**payload)
        raise TypeError("Chunking configuration must be a mapping or ChunkingConfig.")

    def resolved_overlap_tokens(self, chunk_tokens: int | None = None) -> int:
        """Overlap in tokens for a window of ``chunk_tokens`` (fraction rounds down, min 1)."""
        if self.overlap_tokens:
            return int(self.overlap_tokens)
        size = int(chunk_tokens or self.chunk_tokens or 0)
        if size <= 0 or self.overlap_fraction <= 0.0:
            return 0
        return max(1, int(size * self.overlap_fraction))


@dataclass(frozen=True)
class ReferenceChunk:
    """An exact token span of one reference, the unit every PRA layer encodes."""

    chunk_id: str
    source_uri: str
    text: str
    token_ids: tuple[int, ...]
    token_start: int
    token_end: int
    char_start: int | None = None
    char_end: int | None = None
    marker_type: str | None = None
    metadata: dict = field(default_factory=dict)


class ReferencePartitioner(Protocol):
    def partition(self, uri: str, text: str, metadata: dict) -> list[tuple[int, int, str | None]]:
        ...


class SemanticChunker(Protocol):
    def partition(self, uri: str, text: str, token_ids: list[int], metadata: dict,
                  max_chunks: int) -> list[ReferenceChunk]:
        ...


def chunk_identity(uri: str, index: int) -> str:
    """Stable chunk identity shared by every layer's encoding of the span."""
    return f"{uri}#chunk={index}"


class ExplicitMarkerPartitioner:
    """Split at literal markers; with ``retain_markers`` a marker starts the next span."""

    def __init__(self, markers: tuple[str, ...], retain_markers: bool = True):
        self.markers = tuple(m for m in markers if m)
        self.retain_markers = retain_markers

    def partition(self, uri: str, text: str, metadata: dict) -> list[tuple[int, int, str | None]]:
        del uri, metadata
        whole = [(0, len(text), None)] if text else []
        if not self.markers:
            return whole
        pattern = re.compile("|".join(re.escape(m) for m in self.markers))
        cuts = [0]
        found = False
        for match in pattern.finditer(text):
            found = True
            cut = match.start() if self.retain_markers else match.end()
            if cut > cuts[-1]:
                cuts.append(cut)
        if not found:
            return whole
        cuts.append(len(text))
        return [(a, b, "explicit") for a, b in zip(cuts, cuts[1:]) if text[a:b].strip()]


class MarkdownHeadingPartitioner:
    """Markdown headings (``#`` .. ``######``) open new spans; a non-empty preamble is kept."""

    _heading = re.compile(r"(?m)^#{1,6}\s+.+$")

    def partition(self, uri: str, text: str, metadata: dict) -> list[tuple[int, int, str | None]]:
        del uri, metadata
        heads = [m.start() for m in self._heading.finditer(text)]
        if not heads:
            return [(0, len(text), None)] if text else []
        starts = sorted({*heads, *([0] if text[: heads[0]].strip() else [])})
        bounds = starts + [len(text)]
        return [(a, b, "markdown_heading") for a, b in zip(bounds, bounds[1:]) if text[a:b].strip()]


def _spans_to_chunks(uri, text, tokenizer, spans, metadata) -> list[ReferenceChunk]:
    out = []
    for index, (c0, c1, kind) in enumerate(spans):
        ids = tuple(tokenizer.encode(text[c0:c1]))
        if not ids:
            continue
        start = len(tokenizer.encode(text[:c0]))
        out.append(ReferenceChunk(chunk_identity(uri, index), uri, text[c0:c1], ids, start,
                                  start + len(ids), c0, c1, kind, dict(metadata)))
    return out


def _window_chunks(uri, token_ids, tokenizer, metadata, *, size, overlap=0) -> list[ReferenceChunk]:
    """Fixed token windows of ``size`` advancing by ``size - overlap``; the last may be short."""
    n = len(token_ids)
    stride = size - overlap
    out = []
    start = 0
    while start < n:
        stop = min(start + size, n)
        ids = tuple(token_ids[start:stop])
        out.append(ReferenceChunk(
            chunk_identity(uri, len(out)), uri, tokenizer.decode(ids), ids, start, stop,
            metadata={**metadata, "overlap_tokens": overlap, "unique_source_tokens": n},
        ))
        if stop == n:
            break
        start += stride
    return out


def _bound_chunk_lengths(chunks, tokenizer, max_chunk_tokens):
    if max_chunk_tokens is None:
        return chunks
    out: list[ReferenceChunk] = []
    for chunk in chunks:
        if len(chunk.token_ids) <= max_chunk_tokens:
            chunk_id = chunk_identity(chunk.source_uri, len(out))
            out.append(chunk if chunk.chunk_id == chunk_id else replace(chunk, chunk_id=chunk_id))
            continue
        for offset in range(0, len(chunk.token_ids), max_chunk_tokens):
            ids = tuple(chunk.token_ids[offset: offset + max_chunk_tokens])
            out.append(replace(
                chunk,
                chunk_id=chunk_identity(chunk.source_uri, len(out)),
                text=tokenizer.decode(ids),
                token_ids=ids,
                token_start=chunk.token_start + offset,
                token_end=chunk.token_start + offset + len(ids),
                char_start=None,
                char_end=None,
                metadata={**chunk.metadata, "bounded_token_split": True},
            ))
    return out


def _cap_chunks(chunks, max_chunks, policy, all_ids, text, tokenizer):
    if max_chunks is None or len(chunks) <= max_chunks:
        return chunks, 0
    dropped = len(chunks) - max_chunks
    if policy == "error":
        raise ValueError(f"Reference produced {len(chunks)} chunks, exceeding max_gists_per_reference={max_chunks}.")
    if policy == "truncate":
        return chunks[:max_chunks], dropped
    if policy != "merge_tail":
        raise ValueError(f"Unsupported gist overflow policy: {policy}")
    keep = chunks[: max_chunks - 1] if max_chunks > 1 else []
    tail_start = chunks[max_chunks - 1].token_start if max_chunks > 1 else 0
    tail_ids = tuple(all_ids[tail_start:])
    last = chunks[max_chunks - 1]
    merged = replace(
        last,
        chunk_id=chunk_identity(chunks[0].source_uri, max_chunks - 1),
        text=tokenizer.decode(tail_ids) if tail_ids else text,
        token_ids=tail_ids,
        token_start=tail_start,
        token_end=len(all_ids),
        char_end=len(text),
        metadata={**last.metadata, "merged_tail_chunks": dropped + 1},
    )
    return [*keep, merged], dropped


def _union_length(spans) -> int:
    """Number of integer positions covered by half-open [start, end) spans."""
    total, reach = 0, None
    for start, end in sorted(spans):
        if end <= start:
            continue
        if reach is None or start >= reach:
            total += end - start
            reach = end
        elif end > reach:
            total += end - reach
            reach = end
    return total


def partition_source(uri: str, token_ids, tokenizer, chunking, metadata=None, *, text: str | None = None,
                     max_chunks: int | None = None, overflow_policy: str = "truncate",
                     max_chunk_tokens: int | None = None) -> list[ReferenceChunk]:
    """Partition exact token ids with one policy (shared by encoding and routing)."""
    policy = ChunkingConfig.from_value(chunking)
    meta = dict(metadata or {})
    ids = list(map(int, token_ids))
    if not ids:
        return []
    text = tokenizer.decode(ids) if text is None else text

    if policy.mode == "none":
        chunks = [ReferenceChunk(chunk_identity(uri, 0), uri, text, tuple(ids), 0, len(ids), 0, len(text),
                                 metadata=meta)]
    elif policy.mode == "fixed":
        size = int(policy.chunk_tokens or max_chunk_tokens or len(ids))
        chunks = _window_chunks(uri, ids, tokenizer, meta, size=size, overlap=policy.resolved_overlap_tokens(size))
    elif policy.mode == "markers":
        splitter = meta.get("partitioner")
        if splitter is None:
            splitter = (MarkdownHeadingPartitioner() if meta.get("format") == "markdown"
                        else ExplicitMarkerPartitioner(policy.markers))
        chunks = _spans_to_chunks(uri, text, tokenizer, splitter.partition(uri, text, meta), meta)
        rebuilt = tuple(t for c in chunks for t in c.token_ids)
        if rebuilt != tuple(ids):
            size = max_chunk_tokens or policy.chunk_tokens or len(ids)
            chunks = _window_chunks(uri, ids, tokenizer, {**meta, "token_exact_marker_fallback": True}, size=size)
    else:  # semantic
        limit = max_chunks if max_chunks is not None else len(ids)
        chunks = list(policy.semantic_chunker.partition(uri, text, ids, meta, limit))

    chunks = _bound_chunk_lengths(chunks, tokenizer, max_chunk_tokens)
    chunks, dropped = _cap_chunks(chunks, max_chunks, overflow_policy, ids, text, tokenizer)
    if dropped:
        chunks = [replace(c, metadata={**c.metadata, "discarded_chunk_count": dropped}) for c in chunks]
    encoded = sum(len(c.token_ids) for c in chunks)
    covered = _union_length((c.token_start, c.token_end) for c in chunks)
    provenance = {
        "chunk_overlap_fraction": policy.overlap_fraction,
        "resolved_chunk_overlap_tokens": policy.resolved_overlap_tokens(policy.chunk_tokens),
        "encoded_tokens_including_overlap": encoded,
        "stored_kv_tokens_including_overlap": encoded,
        "covered_unique_source_tokens": covered,
        "duplication_factor": encoded / max(covered, 1),
    }
    return [replace(c, metadata={**c.metadata, **provenance}) for c in chunks]


def partition_reference_tokens(uri: str, token_ids, tokenizer, config, metadata=None, *, text: str | None = None,
                               max_chunks: int | None = None, use_configured_max_chunks: bool = True,
                               max_chunk_tokens: int | None = None) -> list[ReferenceChunk]:
    """Partition with the config's routing policy; ``use_configured_max_chunks=False``
    makes ``max_chunks=None`` unlimited (implicit prompt history)."""
    routing = getattr(config, "routing_chunking_config", None)
    if routing is None:
        routing = ChunkingConfig(mode=config.chunking_mode, chunk_tokens=config.fixed_chunk_tokens,
                                 overlap_fraction=config.chunk_overlap_fraction,
                                 overlap_tokens=config.fixed_chunk_overlap_tokens,
                                 markers=tuple(config.marker_rules), semantic_chunker=config.semantic_chunker)
    cap = config.max_gists_per_reference if use_configured_max_chunks else max_chunks
    return partition_source(uri, token_ids, tokenizer, routing, metadata, text=text, max_chunks=cap,
                            overflow_policy=config.gist_overflow_policy, max_chunk_tokens=max_chunk_tokens)


def partition_reference(uri: str, text: str, tokenizer, config, metadata=None) -> list[ReferenceChunk]:
    """Tokenise one resolved text and partition it into routable chunks."""
    return partition_reference_tokens(uri, list(tokenizer.encode(text)), tokenizer, config, metadata, text=text)


__all__ = [
    "ChunkingConfig",
    "ExplicitMarkerPartitioner",
    "MarkdownHeadingPartitioner",
    "ReferenceChunk",
    "ReferencePartitioner",
    "SemanticChunker",
    "chunk_identity",
    "partition_reference",
    "partition_reference_tokens",
    "partition_source",
]
