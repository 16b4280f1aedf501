"""The object path reproduces the reference model exactly on CPU (same weights, fp32)."""

import warnings

import pytest
import torch

from pdattention_b200.config import PRAConfig
from pdattention_b200.data import PRADataModule
from pdattention_b200.data.generators import generate_hierarchy, generate_kv_qa, generate_synthetic
from pdattention_b200.memory import PRABatchedMemoryCache, build_cache_from_metadata, prepare_prompt_batch_for_pra
from pdattention_b200.models import TinyPRAModel, convert_sa_model_to_pra


@pytest.fixture(scope="module")
def stages(tmp_path_factory):
    root = tmp_path_factory.mktemp("data")
    generate_synthetic(root / "stage0_synthetic_memory", n=6)
    generate_hierarchy(root / "stage1_hierarchical_synthetic", n=3)
    generate_kv_qa(root / "synthetic_kv_qa", n=4, min_doc_tokens=60, max_doc_tokens=90)
    return root


def _pair(ref, **kw):
    base = dict(vocab_size=130, d_model=32, n_heads=4, n_layers=3, max_seq_len=128, device="cpu")
    base.update(kw)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        theirs = ref.model.TinyPRAModel(ref.config.PRAConfig(**base)).eval()
        mine = TinyPRAModel(PRAConfig(**base)).eval()
    assert set(theirs.state_dict()) == set(mine.state_dict())
    mine.load_state_dict(theirs.state_dict())
    return mine, theirs


def _batch(stages, stage, n=2, seq=128):
    dm = PRADataModule(stage, str(stages), batch_size=n, max_seq_len=seq, shuffle=False).load()
    return dm.tokenizer, next(iter(dm.test_loader() if False else dm._loader(dm.dataset, shuffle=False)))


def _selections(model):
    return {l: [[(h.chunk_id, round(h.chunk_score, 5)) for h in row] for row in rows]
            for l, rows in model.selected_chunks_by_layer().items()}


VARIANTS = [
    dict(),
    dict(n_vanilla_layers=1, n_mixed_layers=1),
    dict(model_variant="tdx_pra", n_layers=4),
    dict(memory_transport="cross_attention", memory_bucket_count=2),
    dict(chunking_mode="fixed", fixed_chunk_tokens=16, top_k_chunks_per_reference=3, trigger_threshold=-1.0),
    dict(chunking_mode="fixed", fixed_chunk_tokens=16, fixed_chunk_overlap_tokens=4, top_k_chunks_per_reference=3,
         trigger_threshold=-1.0),
    dict(chunking_mode="fixed", fixed_chunk_tokens=16, detail_materialization="gist_only", trigger_threshold=-1.0),
    dict(chunking_mode="fixed", fixed_chunk_tokens=16, detail_materialization="full_reference",
         trigger_threshold=-1.0, max_materialized_memory_tokens=40),
    dict(chunking_mode="fixed", fixed_chunk_tokens=16, search_strategy="global_chunks", trigger_threshold=-1.0,
         gist_mode="kmeans", gists_per_chunk=2),
    dict(chunking_mode="fixed", fixed_chunk_tokens=16, search_strategy="reference_first",
         reference_level_gist_mode="mean", trigger_threshold=-1.0),
]


@pytest.mark.parametrize("variant", VARIANTS)
def test_batched_forward_matches_reference(ref, stages, variant):
    torch.manual_seed(0)
    mine, theirs = _pair(ref, **variant)
    tok, batch = _batch(stages, "stage0_synthetic_memory", n=3)
    mcaches = [build_cache_from_metadata(mine, tok, [m], "cpu", attach_to_model=False) for m in batch["metadata"]]
    rcaches = [ref.cache_services.build_cache_from_metadata(theirs, tok, [m], "cpu", attach_to_model=False)
               for m in batch["metadata"]]
    mine.set_pra_cache(PRABatchedMemoryCache(mcaches))
    theirs.set_pra_cache(ref.memory.PRABatchedMemoryCache(rcaches))
    with torch.no_grad():
        a = mine(batch["input_ids"], attention_mask=batch["attention_mask"])
        b = theirs(batch["input_ids"], attention_mask=batch["attention_mask"])
    assert torch.allclose(a, b, atol=1e-5), (a - b).abs().max()
    assert _selections(mine) == _selections(theirs)
    da, db = mine.pra_diagnostics_by_layer(), theirs.pra_diagnostics_by_layer()
    for layer in da:
        assert set(k for k in da[layer] if k != "batching") == set(k for k in db[layer] if k != "batching")


def test_recursive_build_matches_reference(ref, stages):
    mine, theirs = _pair(ref, recursive_refs_enabled=True, chunking_mode="fixed", fixed_chunk_tokens=16,
                         trigger_threshold=-1.0)
    tok, batch = _batch(stages, "stage1_hierarchical_synthetic", n=2)
    a = build_cache_from_metadata(mine, tok, batch["metadata"][:1], "cpu")
    b = ref.cache_services.build_cache_from_metadata(theirs, tok, batch["metadata"][:1], "cpu")
    assert [(e.uri, e.event, e.depth) for e in a.resolution_events] == \
           [(e.uri, e.event, e.depth) for e in b.resolution_events]
    assert a.dependencies == b.dependencies
    for uri, entry in b.entries.items():
        mine_entry = a.entries[uri]
        for layer, memory in entry.layer_memory.items():
            for ca, cb in zip(mine_entry.layer_memory[layer].chunks, memory.chunks):
                assert torch.allclose(ca.token_kv.k, cb.token_kv.k, atol=1e-5)
                assert torch.allclose(ca.routing_gist.k, cb.routing_gist.k, atol=1e-5)
    with torch.no_grad():
        assert torch.allclose(mine(batch["input_ids"][:1]), theirs(batch["input_ids"][:1]), atol=1e-5)


def test_historical_head_plus_tail_equals_dense(stages):
    """Encoding the head historically and attending natively reproduces the dense forward."""
    cfg = PRAConfig(vocab_size=130, d_model=32, n_heads=4, n_layers=2, max_seq_len=96, model_variant="td_pra",
                    max_prompt_direct_tokens=24, prompt_overflow_mode="implicit_reference",
                    prompt_position_mode="historical", chunking_mode="fixed", fixed_chunk_tokens=16,
                    top_k_references=1, top_k_chunks_per_reference=100, trigger_threshold=-10.0,
                    max_prompt_gists=None, device="cpu")
    torch.manual_seed(3)
    model = TinyPRAModel(cfg).eval()
    ids = torch.randint(1, 120, (1, 70))

    class Tok:
        def decode(self, x):
            return "".join(chr(65 + int(v) % 50) for v in x)

        def encode(self, s):
            return [ord(c) - 65 for c in s]

    with torch.no_grad():
        dense = model(ids, use_pra_memory=False)
        prepared = prepare_prompt_batch_for_pra(model, Tok(), ids)
        model.set_pra_cache(prepared.caches[0])
        tail = model(prepared.input_ids, position_offset=prepared.position_offsets)
    assert torch.allclose(tail[0], dense[0, -24:], atol=2e-5)


def test_sa_conversion_is_exact(ref):
    sa = TinyPRAModel(PRAConfig(vocab_size=50, d_model=32, n_heads=4, n_layers=2, max_seq_len=32,
                                model_variant="td_sa")).eval()
    target = PRAConfig(vocab_size=50, d_model=32, n_heads=4, n_layers=2, max_seq_len=32, model_variant="td_pra")
    pra = convert_sa_model_to_pra(sa, target).eval()
    ids = torch.randint(0, 50, (2, 20))
    with torch.no_grad():
        assert torch.allclose(sa(ids), pra(ids, use_pra_memory=False), atol=1e-5)


def test_generation_rollover_matches_reference(ref, stages):
    kw = dict(max_prompt_direct_tokens=20, prompt_overflow_mode="implicit_reference", chunking_mode="fixed",
              fixed_chunk_tokens=8, trigger_threshold=-1.0, model_variant="td_pra", n_layers=2)
    mine, theirs = _pair(ref, **kw)
    tok, batch = _batch(stages, "stage0_synthetic_memory", n=1)
    ids = batch["input_ids"][:, :30]
    a = mine.generate(ids, max_new_tokens=12, tokenizer=tok, do_sample=False)
    b = theirs.generate(ids, max_new_tokens=12, tokenizer=tok, do_sample=False)
    assert torch.equal(a, b)
    for key in ("rollover_events", "tokens_migrated", "head_tokens", "max_direct_tokens_observed"):
        assert mine.last_generation_stats[key] == theirs.last_generation_stats[key]


def test_checkpoint_loads_in_reference_loader(ref, stages, tmp_path):
    mine, _ = _pair(ref)
    tok, _ = _batch(stages, "stage0_synthetic_memory")
    path = tmp_path / "pra_tiny.pt"
    torch.save({"model": mine.state_dict(), "cfg": mine.cfg.__dict__, "stoi": tok.stoi, "itos": tok.itos}, path)
    import importlib

    ref_eval = importlib.import_module("pra_torch.eval")
    model, _tok, loaded = ref_eval.load_model_and_tokenizer(str(path), "cpu", [])
    assert loaded
    ids = torch.randint(0, 100, (1, 12))
    with torch.no_grad():
        assert torch.allclose(model(ids), mine(ids), atol=1e-6)
