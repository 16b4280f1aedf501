"""Service registry (resolvers, caches) and collator-metadata-to-cache construction.

``create_resolver`` / ``create_cache`` instantiate the backend a service config
names (``ResolverServiceConfig`` / ``CacheServiceConfig``: ``type`` plus keyword
``options``) from a registry that other modules extend with
``register_resolver`` / ``register_cache``; unknown types raise ``ValueError``.
``build_cache_from_metadata`` turns one batch's collator metadata into a ready
cache (the entry point of ``src/pra_torch/cache_services.py:69-130``): the
references each row carries (with the documents they bring along) become the
resolver's documents, and every distinct root URI is built child-first by the
recursive builder, or, for grouped encoding strategies, encoded jointly.
``plan_cache_builds`` runs the same traversal without encoding, for the batched
device encoder.
"""

from __future__ import annotations

from collections.abc import Callable, Iterable

from ..config import CacheServiceConfig, ResolverServiceConfig
from .cache import PRAMemoryCache, PRASimpleMemoryCache
from .prompt import IMPLICIT_PROMPT_HEAD_URI
from .resolution import RecursiveReferenceCacheBuilder
from .resolver import InMemoryResolver

RESOLVERS: dict[str, Callable] = {"in_memory": InMemoryResolver}
CACHES: dict[str, Callable[..., PRAMemoryCache]] = {"simple": PRASimpleMemoryCache}


def register_resolver(name: str, factory: Callable) -> None:
    """Make ``ResolverServiceConfig(type=name)`` build ``factory(documents, summaries, **options)``."""
    RESOLVERS[name] = factory


def register_cache(name: str, factory: Callable[..., PRAMemoryCache]) -> None:
    """Make ``CacheServiceConfig(type=name)`` build ``factory(**options)``."""
    CACHES[name] = factory


def _factory(table: dict, kind: str, name: str):
    try:
        return table[name]
    except KeyError:
        raise ValueError(f"Unsupported {kind} service type: {name}") from None


def create_resolver(config, documents: dict, summaries: dict[str, str] | None = None):
    config = ResolverServiceConfig.from_value(config)
    return _factory(RESOLVERS, "resolver", config.type)(documents, summaries, **config.options)


def create_cache(config) -> PRAMemoryCache:
    config = CacheServiceConfig.from_value(config)
    return _factory(CACHES, "cache", config.type)(**config.options)


_CARRIER_KEYS = frozenset({"text", "reference_table", "documents"})


def _document_from_handle(ref) -> tuple[dict, dict]:
    """(the handle's own document, the documents it carries along)."""
    meta = dict(ref.metadata or {})
    own = {"text": str(meta.get("text", "")), "summary": ref.summary,
           "reference_table": dict(meta.get("reference_table") or {}),
           "metadata": {k: v for k, v in meta.items() if k not in _CARRIER_KEYS}, "version": meta.get("version")}
    return own, dict(meta.get("documents") or {})


def collect_reference_metadata(metadata: Iterable[dict]) -> tuple[dict, dict[str, str], list]:
    """Collator metadata -> (resolver documents, summaries, root handles in order).

    Later definitions of a URI replace earlier ones, in handle order (a handle's
    own document first, then the documents it carries).
    """
    documents: dict = {}
    summaries: dict[str, str] = {}
    handles = [ref for item in metadata for ref in item["references"]]
    for ref in handles:
        if ref.uri == IMPLICIT_PROMPT_HEAD_URI:
            raise ValueError(f"Reference URI {IMPLICIT_PROMPT_HEAD_URI!r} is reserved by PRA.")
        own, carried = _document_from_handle(ref)
        documents[ref.uri] = own
        if ref.summary:
            summaries[ref.uri] = ref.summary
        documents.update((str(uri), value) for uri, value in carried.items())
    return documents, summaries, handles


def _roots(handles) -> list[str]:
    return list(dict.fromkeys(ref.uri for ref in handles))


def _encode_grouped(model, tokenizer, documents, roots, cache, device) -> None:
    if model.cfg.recursive_refs_enabled:
        raise NotImplementedError("Grouped reference encoding is not yet compatible with recursive cache builds.")
    group = [{"uri": uri, "text": str(documents[uri].get("text", "")),
              "metadata": dict(documents[uri].get("metadata") or {})} for uri in roots]
    for entry in model.encode_reference_group_to_cache(group, tokenizer, device):
        cache.put(entry)
    cache.resolution_events, cache.dependencies = [], []


def build_cache_from_metadata(model, tokenizer, metadata: list[dict], device, *, resolver_config=None,
                              cache_config=None, resolver=None, cache: PRAMemoryCache | None = None,
                              attach_to_model: bool = True) -> PRAMemoryCache:
    """Resolve every distinct root URI of ``metadata`` into a ready cache.

    Explicit ``resolver`` / ``cache`` instances override the configs.  With
    ``attach_to_model=False`` the model's previous cache is restored afterwards
    (recursive builds attach the row cache while they run, so a parent can read
    its finished children).
    """
    documents, summaries, handles = collect_reference_metadata(metadata)
    resolver = resolver if resolver is not None else create_resolver(resolver_config, documents, summaries)
    cache = cache if cache is not None else create_cache(cache_config)
    roots = _roots(handles)
    if model.cfg.reference_encoding_strategy != "independent":
        _encode_grouped(model, tokenizer, documents, roots, cache, device)
    else:
        previous = model.pra_cache
        builder = RecursiveReferenceCacheBuilder(model, resolver, tokenizer, cache, model.cfg)
        try:
            for uri in roots:
                builder.ensure_cached(uri)
        finally:
            if not attach_to_model:
                model.set_pra_cache(previous)
        cache.resolution_events, cache.dependencies = list(builder.events), list(builder.dependencies)
    if attach_to_model:
        model.set_pra_cache(cache)
    return cache


def plan_cache_builds(model, tokenizer, metadata_rows: list[dict], *, resolver_config=None):
    """Per row: a fresh cache and a planning-mode builder that traversed the row's roots
    (its ``plan`` lists the encodes in order, with their visible entries)."""
    caches, builders = [], []
    for item in metadata_rows:
        documents, summaries, handles = collect_reference_metadata([item])
        cache = PRASimpleMemoryCache()
        builder = RecursiveReferenceCacheBuilder(model, create_resolver(resolver_config, documents, summaries),
                                                 tokenizer, cache, model.cfg, plan_only=True)
        for uri in _roots(handles):
            builder.ensure_cached(uri)
        caches.append(cache)
        builders.append(builder)
    return caches, builders


# Device caches of the Llama-family engine: ``CacheServiceConfig(type="paged", options={...})``
# builds a deduplicated device page pool (``inference.page_cache.PagedChunkCache``) bound to an
# engine; options: ``capacity_pages``, ``host_capacity_pages``, ``chunk_tokens``.
DEVICE_CACHES: dict[str, Callable] = {}


def register_device_cache(name: str, factory: Callable) -> None:
    """Make ``create_device_cache(engine, CacheServiceConfig(type=name))`` build ``factory(engine, **options)``."""
    DEVICE_CACHES[name] = factory


def create_device_cache(engine, config: CacheServiceConfig | dict | None = None):
    config = CacheServiceConfig.from_value(config) if config is not None else CacheServiceConfig(type="paged")
    if config.type not in DEVICE_CACHES and config.type == "paged":
        from ..inference.page_cache import PagedChunkCache

        register_device_cache("paged", PagedChunkCache)
    return _factory(DEVICE_CACHES, "device cache", config.type)(engine, **dict(config.options or {}))
