import math
from types import SimpleNamespace

import pytest
import torch

from pdattention_b200.config import PRAConfig
from pdattention_b200.memory import (CacheBuildState, ChunkRoutingGist, LayerKV, LayerReferenceMemory,
                                     PRABatchedMemoryCache, PRACacheEntry, PRASimpleMemoryCache,
                                     ReferenceChunkMemory)
from pdattention_b200.memory.gists import compute_gists, kmeanspp_random_stream


def _entries(mod, n_refs=4, chunks=(3, 12, 2, 5), g=2, d=8, seed=0):
    gen = torch.Generator().manual_seed(seed)
    out = []
    for r in range(n_refs):
        entry = mod.PRACacheEntry(uri=f"mem://ref{(r * 7) % n_refs}", text="t")
        mem = mod.LayerReferenceMemory()
        for c in range(chunks[r]):
            kv = torch.randn(1, 2, 3 + c % 2, d // 2, generator=gen)
            gist = torch.randn((1 + (c % g)), d, generator=gen)
            mem.chunks.append(mod.ReferenceChunkMemory(f"{entry.uri}#chunk={c}", entry.uri, 4 * c, 4 * c + 3,
                                                       mod.LayerKV(kv, kv.clone()), mod.ChunkRoutingGist(k=gist)))
        entry.layer_memory[0] = mem
        out.append(entry)
    return out


def _fill(cache_cls, mod, **kw):
    cache = cache_cls()
    for e in _entries(mod, **kw):
        cache.put(e)
    return cache


STRATEGIES = [
    dict(search_strategy="hierarchical"), dict(search_strategy="global_chunks"),
    dict(search_strategy="reference_first", reference_level_gist_mode="mean"),
]


@pytest.mark.parametrize("strategy", STRATEGIES)
@pytest.mark.parametrize("backend", ["tensorized", "legacy"])
@pytest.mark.parametrize("agg", ["max", "mean", "logsumexp"])
@pytest.mark.parametrize("rankings", [False, True])
def test_search_matches_reference(ref, strategy, backend, agg, rankings):
    import pdattention_b200.memory.cache as mine_mod

    kw = dict(top_k_references=2, top_k_chunks_per_reference=3, routing_backend=backend, gist_score_aggregation=agg,
              reference_score_aggregation=agg, collect_routing_metrics=rankings, **strategy)
    mine = _fill(PRASimpleMemoryCache, mine_mod)
    theirs = _fill(ref.memory.PRASimpleMemoryCache, ref.memory)
    q = torch.randn(3, 8, generator=torch.Generator().manual_seed(5))
    a = mine.search(q, 0, PRAConfig(**kw))
    b = theirs.search(q, 0, ref.config.PRAConfig(**kw))
    fields = ("reference_uri", "chunk_id", "reference_rank", "rank_within_reference", "winning_gist_index",
              "gist_count")
    assert [[tuple(getattr(h, f) for f in fields) for h in row] for row in a] == \
           [[tuple(getattr(h, f) for f in fields) for h in row] for row in b]
    for ra, rb in zip(a, b):
        for ha, hb in zip(ra, rb):
            assert math.isclose(ha.chunk_score, hb.chunk_score, rel_tol=1e-5, abs_tol=1e-6)
            assert math.isclose(ha.reference_score, hb.reference_score, rel_tol=1e-5, abs_tol=1e-6)
    if rankings:
        _assert_close(mine.last_rankings(0), theirs.last_rankings(0))


def _assert_close(a, b):
    if isinstance(a, dict):
        assert a.keys() == b.keys()
        for key in a:
            _assert_close(a[key], b[key])
    elif isinstance(a, (list, tuple)):
        assert len(a) == len(b)
        for x, y in zip(a, b):
            _assert_close(x, y)
    elif isinstance(a, float):
        assert math.isclose(a, b, rel_tol=1e-5, abs_tol=1e-6)
    else:
        assert a == b


def test_lexical_chunk_tie_break_is_not_numeric():
    import pdattention_b200.memory.cache as m

    cache = PRASimpleMemoryCache()
    entry = PRACacheEntry(uri="u", text="")
    mem = LayerReferenceMemory()
    gist = torch.ones(1, 4)
    for c in (2, 10):
        kv = torch.zeros(1, 1, 2, 4)
        mem.chunks.append(ReferenceChunkMemory(f"u#chunk={c}", "u", c, c + 1, LayerKV(kv, kv), ChunkRoutingGist(k=gist)))
    entry.layer_memory[0] = mem
    cache.put(entry)
    hits = cache.search(torch.ones(1, 4), 0, PRAConfig(top_k_references=1, top_k_chunks_per_reference=2))[0]
    assert [h.chunk_id for h in hits] == ["u#chunk=10", "u#chunk=2"]
    del m


def test_lifecycle_and_batched_isolation():
    cache = PRASimpleMemoryCache()
    cache.begin_build("a")
    assert cache.state("a") == CacheBuildState.BUILDING and cache.get("a") is None and cache.is_empty()
    cache.mark_failed("a", RuntimeError("boom"))
    assert cache.state("a") == CacheBuildState.FAILED and cache.failure("a") == "boom"
    import pdattention_b200.memory.cache as m

    full = _fill(PRASimpleMemoryCache, m)
    batched = PRABatchedMemoryCache([full, PRASimpleMemoryCache()])
    rows = batched.search(torch.randn(2, 8), 0, PRAConfig())
    assert rows[0] and rows[1] == []
    with pytest.raises(RuntimeError):
        batched.get("x")
    with pytest.raises(ValueError):
        batched.search(torch.randn(3, 8), 0, PRAConfig())


def test_prepare_routing_index_reports_reuse():
    import pdattention_b200.memory.cache as m

    cache = _fill(PRASimpleMemoryCache, m)
    q = torch.randn(8)
    first = cache.prepare_routing_index(0, q)
    second = cache.prepare_routing_index(0, q)
    assert not first["reused"] and second["reused"] and second["candidate_chunks"] == 22


GIST_CASES = [("mean", 1, {}), ("last", 1, {}), ("kmeans", 2, {}), ("kmeans", 4, {"gist_kmeans_init": "sample"}),
              ("kmeans", 3, {"gist_kmeans_normalize": False}), ("som", 3, {}), ("prototype", 3, {}),
              ("prototype", 2, {"gist_prototype_init": "sample", "gist_prototype_refine": False}),
              ("hybrid", 3, {}), ("hybrid", 3, {"gist_hybrid_local_mode": "som"})]


@pytest.mark.parametrize("mode,count,extra", GIST_CASES)
def test_gists_match_reference(ref, mode, count, extra):
    keys = torch.randn(17, 12, generator=torch.Generator().manual_seed(1))
    values = torch.randn(17, 12, generator=torch.Generator().manual_seed(2))
    cfg = PRAConfig(**extra)
    rcfg = ref.config.PRAConfig(**extra)
    a = compute_gists(keys=keys, values=values, mode=mode, num_gists=count, config=cfg,
                      context=SimpleNamespace(token_ids=(), tokenizer=None, ref_end_token="<REF_END>",
                                              gru_pooler=None, level="chunk"))
    b = ref.gists.compute_gists(keys=keys, values=values, mode=mode, num_gists=count, config=rcfg,
                                context=ref.gists.GistContext(level="chunk"))
    assert torch.allclose(a.k, b.k, atol=1e-6) and torch.allclose(a.v, b.v, atol=1e-6)
    assert a.metadata.get("occupancy") == b.metadata.get("occupancy")


def test_kmeanspp_stream_reproduces_generator():
    first, draws = kmeanspp_random_stream(64, 3, seed=0)
    gen = torch.Generator().manual_seed(0)
    assert first == int(torch.randint(64, (1,), generator=gen).item())
    p = torch.rand(64)
    p = p / p.sum()
    assert int(torch.multinomial(p, 1, generator=gen).item()) == int(torch.argmax(p / draws[0]).item())
