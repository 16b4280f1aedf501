"""Memory services: cache data model and lifecycle, routing, gists, chunking glue,
resolver, recursive builder, prompt heads and the batched/paged device store."""

from .batching import MemoryBatchingStats, MemoryBucket, MemoryBucketPlanner, dynamic_memory_attention, \
    native_kv_attention, padded_memory_attention
from .cache import (
    CacheBuildState,
    ChunkKV,
    ChunkRoutingGist,
    LayerKV,
    LayerReferenceMemory,
    PRABatchedMemoryCache,
    PRACacheEntry,
    PRAMemoryCache,
    PRASimpleMemoryCache,
    ReferenceChunkMemory,
    ReferenceRoutingGists,
    RoutingIndex,
    SelectedChunk,
)
from .prompt import IMPLICIT_PROMPT_HEAD_NAME, IMPLICIT_PROMPT_HEAD_URI, prepare_prompt_batch_for_pra, \
    prepare_prompt_for_pra
from .resolution import RecursiveReferenceCacheBuilder, ResolutionBudget, ResolutionBudgetExceeded, ResolutionEvent
from .resolver import InMemoryResolver, ResolvedReference
from .services import build_cache_from_metadata, collect_reference_metadata, create_cache, create_resolver

__all__ = [name for name in dir() if not name.startswith("_")]
