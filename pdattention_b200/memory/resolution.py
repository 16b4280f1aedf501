"""Bounded child-first recursive cache construction (``src/pra_torch/resolution.py``).

``ensure_cached`` is a depth-first traversal: cycles are detected on the
ancestry path (policy ``skip`` / ``error`` / ``link_only``), re-entry through
the ``BUILDING`` state, missing URIs follow ``skip`` / ``warn`` / ``error``.  A
cached entry is reused only when its content, model, tokenizer and routing
fingerprints (sha256 of sorted JSON) all match.  One shared budget is charged
per root traversal; children are built before the parent, which is published
atomically, and a failure marks the URI ``FAILED`` and re-raises.

The builder can also run in *planning* mode (``plan_only=True``): it performs the
same traversal and fingerprinting but records, instead of encoding, one
``BuildStep`` per entry with the set of entries that would be visible to that
encode.  The batched device encoder executes such plans wave by wave.
"""

from __future__ import annotations

import hashlib
import json
import warnings
from dataclasses import asdict, dataclass, field

from .cache import CacheBuildState, PRACacheEntry, PRAMemoryCache


class ResolutionBudgetExceeded(RuntimeError):
    pass


@dataclass
class ResolutionBudget:
    max_total_references: int
    max_total_tokens: int
    references_used: int = 0
    tokens_used: int = 0

    def consume(self, token_count: int) -> None:
        if self.references_used + 1 > self.max_total_references:
            raise ResolutionBudgetExceeded("max_total_references exhausted")
        if self.tokens_used + token_count > self.max_total_tokens:
            raise ResolutionBudgetExceeded("max_total_tokens exhausted")
        self.references_used += 1
        self.tokens_used += token_count


@dataclass(frozen=True)
class ResolutionEvent:
    uri: str
    event: str
    depth: int
    parent_uri: str | None = None
    detail: str | None = None


@dataclass
class BuildStep:
    """One entry encode in traversal order (planning mode)."""

    uri: str
    text: str
    metadata: dict
    use_pra_memory: bool
    visible_uris: tuple[str, ...]
    depth: int
    token_ids: tuple[int, ...] | None = None  # the text's ids, tokenised once while planning


def _fingerprint(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, default=str).encode("utf-8")).hexdigest()


_VOCAB_FINGERPRINTS: dict[int, tuple[int, object, str]] = {}


def tokenizer_fingerprint(tokenizer) -> str:
    """sha256 of the vocabulary, memoised per tokenizer object and vocabulary size.

    Hashing a large vocabulary on every resolve dominated cache-build time; the
    value only changes when tokens are added, which changes the size.
    """
    stoi = getattr(tokenizer, "stoi", {})
    key = id(tokenizer)
    cached = _VOCAB_FINGERPRINTS.get(key)
    if cached is not None and cached[0] == len(stoi) and cached[1] is tokenizer:
        return cached[2]
    value = _fingerprint(stoi)
    _VOCAB_FINGERPRINTS[key] = (len(stoi), tokenizer, value)
    return value


_ROUTING_IDENTITY_KEYS = {
    "chunking_mode", "fixed_chunk_tokens", "fixed_chunk_overlap_tokens", "max_gists_per_reference", "use_summary",
    "summary_mode", "recursive_refs_enabled", "recursive_max_depth",
}
_ROUTING_IDENTITY_PREFIXES = ("gist_", "gists_", "reference_gist", "reference_level_gist")


class RecursiveReferenceCacheBuilder:
    def __init__(self, model, resolver, tokenizer, cache: PRAMemoryCache, config, *, plan_only: bool = False):
        self.model = model
        self.resolver = resolver
        self.tokenizer = tokenizer
        self.cache = cache
        self.config = config
        self.plan_only = plan_only
        self.events: list[ResolutionEvent] = []
        self.dependencies: list[dict] = []
        self.plan: list[BuildStep] = []
        self._planned_ready: list[str] = []

    def new_budget(self) -> ResolutionBudget:
        return ResolutionBudget(self.config.recursive_max_total_references, self.config.recursive_max_total_tokens)

    def _identity(self, resolved) -> dict:
        if getattr(self, "_static_identity", None) is None:
            routing = {k: v for k, v in asdict(self.config).items()
                       if k.startswith(_ROUTING_IDENTITY_PREFIXES) or k in _ROUTING_IDENTITY_KEYS}
            self._static_identity = (
                _fingerprint({"class": type(self.model).__name__, "d_model": self.config.d_model,
                              "n_layers": self.config.n_layers, "n_heads": self.config.n_heads}),
                _fingerprint(routing))
        model_fp, routing_fp = self._static_identity
        return {
            "canonical_uri": resolved.uri,
            "content_fingerprint": _fingerprint({"text": resolved.text, "version": resolved.version}),
            "model_fingerprint": model_fp,
            "tokenizer_fingerprint": tokenizer_fingerprint(self.tokenizer),
            "routing_configuration_fingerprint": routing_fp,
        }

    def _missing(self, uri: str, depth: int, error: Exception):
        self.events.append(ResolutionEvent(uri, "missing", depth, detail=str(error)))
        policy = self.config.recursive_missing_ref_policy
        if policy == "error":
            raise error
        if policy == "warn":
            warnings.warn(str(error), RuntimeWarning, stacklevel=3)
        return None

    # planning-mode views of the cache
    def _state(self, uri: str):
        if self.plan_only and uri in self._planned_ready:
            return CacheBuildState.READY
        return self.cache.state(uri) if hasattr(self.cache, "state") else CacheBuildState.MISSING

    def _has(self, uri: str) -> bool:
        return (self.plan_only and uri in self._planned_ready) or self.cache.has(uri)

    def ensure_cached(self, uri: str, *, depth: int = 0, ancestry: tuple[str, ...] = (),
                      budget: ResolutionBudget | None = None, parent_uri: str | None = None) -> PRACacheEntry | None:
        budget = budget or self.new_budget()
        cfg = self.config
        if uri in ancestry:
            self.dependencies.append({"parent_uri": parent_uri, "child_uri": uri, "cyclic": True,
                                      "action": cfg.recursive_cycle_policy})
            self.events.append(ResolutionEvent(uri, "cycle", depth, parent_uri=parent_uri))
            if cfg.recursive_cycle_policy == "error":
                raise RuntimeError(f"Recursive reference cycle detected: {' -> '.join((*ancestry, uri))}")
            return self.cache.get(uri) if cfg.recursive_cycle_policy == "link_only" else None
        if self._state(uri) == CacheBuildState.BUILDING:
            self.events.append(ResolutionEvent(uri, "reentrant", depth, parent_uri=parent_uri))
            if cfg.recursive_cycle_policy == "error":
                raise RuntimeError(f"Re-entrant reference cache construction for {uri}")
            return None
        try:
            resolved = self.resolver.resolve(uri)
        except KeyError as error:
            return self._missing(uri, depth, error)

        identity = self._identity(resolved)
        if self.plan_only and uri in self._planned_ready:
            self.events.append(ResolutionEvent(uri, "cache_hit", depth, parent_uri=parent_uri))
            return None
        existing = self.cache.get(uri)
        if existing is not None and all(existing.metadata.get(k) == v for k, v in identity.items()):
            self.events.append(ResolutionEvent(uri, "cache_hit", depth, parent_uri=parent_uri))
            return existing
        if existing is not None and hasattr(self.cache, "invalidate"):
            self.cache.invalidate(uri)

        token_ids = self.tokenizer.encode(resolved.text)
        budget.consume(len(token_ids))
        if hasattr(self.cache, "begin_build") and not self.plan_only:
            self.cache.begin_build(uri)
        self.events.append(ResolutionEvent(uri, "building", depth, parent_uri=parent_uri))
        children = list(dict.fromkeys(resolved.reference_table.values()))[: cfg.recursive_max_children_per_reference]
        try:
            if cfg.recursive_refs_enabled and depth < cfg.recursive_max_depth:
                for child in children:
                    self.dependencies.append({"parent_uri": uri, "child_uri": child, "cyclic": False,
                                              "action": "resolve"})
                    try:
                        self.ensure_cached(child, depth=depth + 1, ancestry=(*ancestry, uri), budget=budget,
                                           parent_uri=uri)
                    except ResolutionBudgetExceeded as error:
                        self.events.append(ResolutionEvent(child, "budget_exhausted", depth + 1, uri, str(error)))
                        break
            elif children:
                reason = "max_depth" if cfg.recursive_refs_enabled else "recursion_disabled"
                for child in children:
                    self.dependencies.append({"parent_uri": uri, "child_uri": child, "cyclic": False,
                                              "action": reason})
            metadata = {**resolved.metadata, **identity, "version": resolved.version, "summary": resolved.summary,
                        "reference_table": resolved.reference_table, "child_uris": children,
                        "resolution_depth": depth, "resolution_budget_references_used": budget.references_used,
                        "resolution_budget_tokens_used": budget.tokens_used}
            use_memory = cfg.recursive_refs_enabled and any(self._has(c) for c in children)
            if self.plan_only:
                ready = [e.uri for e in self.cache.all_entries()] + self._planned_ready
                visible = tuple(dict.fromkeys(ready)) if use_memory else ()
                self.plan.append(BuildStep(uri, resolved.text, metadata, use_memory, visible, depth,
                                           tuple(token_ids)))
                self._planned_ready.append(uri)
                self.events.append(ResolutionEvent(uri, "ready", depth, parent_uri=parent_uri))
                return None
            self.model.set_pra_cache(self.cache)
            entry = self.model.encode_reference_to_cache(uri, resolved.text, self.tokenizer,
                                                         next(self.model.parameters()).device, metadata=metadata,
                                                         use_pra_memory=use_memory)
            self.cache.put(entry)
            self.events.append(ResolutionEvent(uri, "ready", depth, parent_uri=parent_uri))
            return entry
        except Exception as error:
            if hasattr(self.cache, "mark_failed") and not self.plan_only:
                self.cache.mark_failed(uri, error)
            self.events.append(ResolutionEvent(uri, "failed", depth, parent_uri, str(error)))
            raise
