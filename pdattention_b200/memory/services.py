"""Resolver / cache factories and metadata-to-cache construction (``src/pra_torch/cache_services.py``)."""

from __future__ import annotations

from collections.abc import Iterable

from ..config import CacheServiceConfig, ResolverServiceConfig
from .cache import PRAMemoryCache, PRASimpleMemoryCache
from .prompt import IMPLICIT_PROMPT_HEAD_URI
from .resolution import RecursiveReferenceCacheBuilder
from .resolver import InMemoryResolver

RESOLVERS = {"in_memory": InMemoryResolver}
CACHES = {"simple": PRASimpleMemoryCache, "paged": PRASimpleMemoryCache}


def create_resolver(config, documents: dict, summaries: dict[str, str] | None = None):
    config = ResolverServiceConfig.from_value(config)
    if config.type not in RESOLVERS:
        raise ValueError(f"Unsupported resolver service type: {config.type}")
    return RESOLVERS[config.type](documents, summaries, **config.options)


def create_cache(config) -> PRAMemoryCache:
    config = CacheServiceConfig.from_value(config)
    if config.type not in CACHES:
        raise ValueError(f"Unsupported cache service type: {config.type}")
    return CACHES[config.type](**config.options)


def collect_reference_metadata(metadata: Iterable[dict]) -> tuple[dict, dict[str, str], list]:
    """Collator metadata -> (resolver documents, summaries, root handles)."""
    documents: dict = {}
    summaries: dict[str, str] = {}
    handles = []
    for item in metadata:
        for ref in item["references"]:
            if ref.uri == IMPLICIT_PROMPT_HEAD_URI:
                raise ValueError(f"Reference URI {IMPLICIT_PROMPT_HEAD_URI!r} is reserved by PRA.")
            meta = dict(ref.metadata or {})
            documents[ref.uri] = {
                "text": str(meta.get("text", "")), "summary": ref.summary,
                "reference_table": dict(meta.get("reference_table") or {}),
                "metadata": {k: v for k, v in meta.items() if k not in {"text", "reference_table", "documents"}},
                "version": meta.get("version"),
            }
            if ref.summary:
                summaries[ref.uri] = ref.summary
            for child_uri, child in dict(meta.get("documents") or {}).items():
                documents[str(child_uri)] = child
            handles.append(ref)
    return documents, summaries, handles


def build_cache_from_metadata(model, tokenizer, metadata: list[dict], device, *, resolver_config=None,
                              cache_config=None, resolver=None, cache: PRAMemoryCache | None = None,
                              attach_to_model: bool = True) -> PRAMemoryCache:
    """Resolve every distinct root URI of ``metadata`` into a ready cache."""
    documents, summaries, handles = collect_reference_metadata(metadata)
    resolver = resolver if resolver is not None else create_resolver(resolver_config, documents, summaries)
    cache = cache if cache is not None else create_cache(cache_config)
    roots = list(dict.fromkeys(ref.uri for ref in handles))
    if model.cfg.reference_encoding_strategy != "independent":
        if model.cfg.recursive_refs_enabled:
            raise NotImplementedError("Grouped reference encoding is not yet compatible with recursive cache builds.")
        grouped = [{"uri": u, "text": str(documents[u].get("text", "")),
                    "metadata": dict(documents[u].get("metadata") or {})} for u in roots]
        for entry in model.encode_reference_group_to_cache(grouped, tokenizer, device):
            cache.put(entry)
        cache.resolution_events, cache.dependencies = [], []
        if attach_to_model:
            model.set_pra_cache(cache)
        return cache
    previous = model.pra_cache
    builder = RecursiveReferenceCacheBuilder(model, resolver, tokenizer, cache, model.cfg)
    try:
        for uri in roots:
            builder.ensure_cached(uri)
    finally:
        if not attach_to_model:
            model.set_pra_cache(previous)
    cache.resolution_events = list(builder.events)
    cache.dependencies = list(builder.dependencies)
    if attach_to_model:
        model.set_pra_cache(cache)
    return cache


def plan_cache_builds(model, tokenizer, metadata_rows: list[dict], *, resolver_config=None):
    """Traverse every row's references in planning mode (no encoding).

    Returns ``(caches, builders)``: one fresh cache and one builder (holding the
    ordered ``BuildStep`` plan and the audit trail) per row.
    """
    caches, builders = [], []
    for item in metadata_rows:
        documents, summaries, handles = collect_reference_metadata([item])
        resolver = create_resolver(resolver_config, documents, summaries)
        cache = PRASimpleMemoryCache()
        builder = RecursiveReferenceCacheBuilder(model, resolver, tokenizer, cache, model.cfg, plan_only=True)
        for uri in dict.fromkeys(ref.uri for ref in handles):
            builder.ensure_cached(uri)
        caches.append(cache)
        builders.append(builder)
    return caches, builders
