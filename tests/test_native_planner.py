"""The native cache-build planner (csrc/planner.cpp) against the Python planner it replaces.

Both plan the same batches; every output the device encoder reads (waves, encode
sequence numbers, packed wave tables, routing namespaces, chunk tables) and every
record and audit entry must be identical.  Runs on CPU: planning needs no GPU.
"""

import copy

import numpy as np
import pytest

from pdattention_b200.config import PRAConfig, ResolverServiceConfig
from pdattention_b200.core.references import ReferenceHandle
from pdattention_b200.data import WordIdTokenizer
from pdattention_b200.data.tokenizer import PRATokenizer
from pdattention_b200.models import TinyPRAModel
from pdattention_b200.models.fastpath import DeviceRuntime, Namespace
from pdattention_b200.ops import _ext


@pytest.fixture(scope="module", autouse=True)
def _built():
    ext = _ext.load()
    if ext is None or not hasattr(ext, "plan_batch"):
        pytest.skip("extension not built")


def _cfg(**over):
    base = dict(vocab_size=600, d_model=32, n_heads=2, n_layers=1, max_seq_len=128, model_variant="td_pra",
                chunking_mode="fixed", fixed_chunk_tokens=8, top_k_references=2, top_k_chunks_per_reference=2,
                gist_mode="kmeans", gists_per_chunk=2, recursive_refs_enabled=True, recursive_max_depth=2,
                recursive_missing_ref_policy="skip", trigger_threshold=-1.0, device="cpu")
    base.update(over)
    return PRAConfig(**base)


def _words(rng, n, vocab=500):
    return " ".join(f"t{rng.randrange(1, vocab)}" for _ in range(n))


def _doc(text, children=()):
    return {"text": text, "reference_table": {f"<REF_{i + 1}>": c for i, c in enumerate(children)}}


def _row(roots, docs):
    """roots: [(uri, text, children)], docs: {uri: value} carried by the first root's metadata."""
    refs = []
    for i, (uri, text, children) in enumerate(roots):
        meta = {"text": text, "reference_table": {f"<REF_{j + 1}>": c for j, c in enumerate(children)}}
        if i == 0:
            meta["documents"] = docs
        refs.append(ReferenceHandle(id=i + 1, token=f"<REF_{i + 1}>", uri=uri, metadata=meta))
    return {"references": refs}


def _batches():
    import random

    rng = random.Random(0)
    tree = []
    for e in range(3):  # depth-2 trees like the training benchmark
        docs, roots = {}, []
        for r in range(2):
            root = f"tree://e{e}/r{r}"
            child = f"{root}/c0"
            leaves = [f"{child}/g{g}" for g in range(3)]
            for leaf in leaves:
                docs[leaf] = _doc("<REF_1> " + _words(rng, rng.randrange(5, 30)) if False else _words(rng, rng.randrange(5, 30)))
            docs[child] = _doc(_words(rng, 17), leaves)
            roots.append((root, _words(rng, 20), [child]))
        tree.append(_row(roots, docs))
    edge = [
        # a cycle (a -> b -> a), a missing child, a duplicated root, an anchored URI
        _row([("x://a", _words(rng, 12), ["x://b", "x://missing"]), ("x://a", _words(rng, 3), []),
              ("x://c#sec", _words(rng, 9), ["x://a"])],
             {"x://b": _doc(_words(rng, 10), ["x://a"]), "x://c": _doc(_words(rng, 11))}),
        # empty text, plain-string documents, a document redefined by a later root
        _row([("y://e", "", ["y://s"]), ("y://s", _words(rng, 6), [])], {"y://s": "t5 t6 t7 t8 t9 t10 t11 t12 t13"}),
        # many children (max_children cut) and long texts (chunk cap / merge)
        _row([("z://root", _words(rng, 40), [f"z://k{i}" for i in range(12)])],
             {f"z://k{i}": _doc(_words(rng, 25 + i)) for i in range(12)}),
    ]
    return [tree, edge]


def _slice(packed, table, name):
    off, words, count = table[name]
    if name == "valid":
        return packed[off: off + words].view(np.uint8)[:count].tolist()
    return packed[off: off + words].tolist()


def _compare(rt, rows, tok, resolver=None):
    native = rt.plan_native(rows, tok, resolver)
    assert native is not None
    python = rt.plan_batch(copy.deepcopy(rows), tok, resolver)
    assert native.seq_len == python.seq_len
    assert native.waves == python.waves
    assert native.rows == python.rows
    assert len(native.entries) == len(python.entries) and len(native.chunks) == len(python.chunks)
    for a, b in zip(native.entries, python.entries):
        assert (a.row, a.uri, a.text, a.use_memory, tuple(a.visible), list(a.chunks), a.wave) == \
               (b.row, b.uri, b.text, b.use_memory, tuple(b.visible), list(b.chunks), b.wave)
        assert a.metadata == b.metadata
    for a, b in zip(native.chunks, python.chunks):
        assert (a.row, a.entry, a.uri, a.chunk_id, a.token_start, a.token_end, tuple(a.token_ids), a.seq) == \
               (b.row, b.entry, b.uri, b.chunk_id, b.token_start, b.token_end, tuple(b.token_ids), b.seq)
        assert a.metadata == b.metadata
    for tn, tp in zip(native.wave_tables, python.wave_tables):
        names = [k for k, v in tp.items() if isinstance(v, tuple)]
        assert sorted(names) == sorted(k for k, v in tn.items() if isinstance(v, tuple))
        for name in names:
            assert _slice(native.packed, tn, name) == _slice(python.packed, tp, name), name
        for key in ("n", "max_len", "has_ns"):
            assert tn[key] == tp[key], key
        if tp["has_ns"]:
            assert tn["ns_empty"] == tp["ns_empty"]
    for bn, bp in zip(native.builders, python.builders):
        assert bn.events == bp.events
        assert bn.dependencies == bp.dependencies
    prompt = Namespace.host_arrays(python.rows, python.entries, python.chunks)
    for i, arr in enumerate(prompt):
        assert _slice(native.packed, native.prompt_table, f"ns{i}") == (arr or [0])
    chunks = python.chunks
    for name, values in (("chunk_start", [c.token_start for c in chunks]), ("chunk_len", [len(c.token_ids) for c in chunks]),
                         ("chunk_pool_row", [c.seq * python.seq_len for c in chunks])):
        assert _slice(native.packed, native.prompt_table, name) == (values or [0])
    return native


@pytest.mark.parametrize("over", [
    {},
    {"gist_mode": "mean", "gists_per_chunk": 1},
    {"fixed_chunk_overlap_tokens": 3},
    {"max_gists_per_reference": 2, "gist_overflow_policy": "truncate"},
    {"max_gists_per_reference": 2, "gist_overflow_policy": "merge_tail"},
    {"recursive_max_depth": 1},
    {"recursive_refs_enabled": False},
    {"recursive_max_children_per_reference": 3},
    {"recursive_max_total_references": 5},
    {"recursive_max_total_tokens": 90},
    {"recursive_cycle_policy": "link_only"},
    {"context_safety_reserve_tokens": 4, "max_materialized_memory_tokens": 50},
])
@pytest.mark.parametrize("layer_sync", [True, False])
def test_native_plan_equals_python_plan(over, layer_sync, monkeypatch):
    from pdattention_b200.models import fastpath

    monkeypatch.setattr(fastpath, "_LAYER_SYNC", layer_sync)
    cfg = _cfg(**over)
    rt = DeviceRuntime.for_planning(TinyPRAModel(cfg))
    tok = WordIdTokenizer(500, [f"<REF_{i}>" for i in range(1, 20)])
    for rows in _batches():
        _compare(rt, rows, tok, ResolverServiceConfig())


def test_python_tokenizers_go_through_their_encode():
    cfg = _cfg(max_seq_len=1024, fixed_chunk_tokens=16)
    rt = DeviceRuntime.for_planning(TinyPRAModel(cfg))
    tok = PRATokenizer()
    rows = [_row([("c://a", "hello world, a plain text", ["c://b"])], {"c://b": "short child text"})]
    _compare(rt, rows, tok)


def test_cases_the_native_planner_hands_back():
    tok = WordIdTokenizer(500, ["<REF_1>"])
    rows = [_row([("w://a", "t1 t2", ["w://missing"])], {})]
    warn = DeviceRuntime.for_planning(TinyPRAModel(_cfg(recursive_missing_ref_policy="warn")))
    assert warn.plan_native(rows, tok) is None  # the Python planner warns
    unregistered = [_row([("w://b", "t1 <REF_77> t3", [])], {})]
    skip = DeviceRuntime.for_planning(TinyPRAModel(_cfg()))
    assert skip.plan_native(unregistered, tok) is None  # the Python tokenizer registers the token
    over_budget = DeviceRuntime.for_planning(TinyPRAModel(_cfg(recursive_max_total_tokens=1)))
    assert over_budget.plan_native([_row([("w://c", "t1 t2 t3", [])], {})], tok) is None


def test_later_document_definitions_replace_earlier_ones():
    """A later reference's document map may redefine an earlier root or another map's entry."""
    import random

    rng = random.Random(3)
    first = {"o://shared": _doc(_words(rng, 9)), "o://r1": _doc(_words(rng, 4))}
    second = {"o://shared": _doc(_words(rng, 13)), "o://r0": "t7 t8 t9"}
    refs = [ReferenceHandle(id=1, token="<REF_1>", uri="o://r0",
                            metadata={"text": _words(rng, 12), "reference_table": {"<REF_9>": "o://shared"},
                                      "documents": first}),
            ReferenceHandle(id=2, token="<REF_2>", uri="o://r1",
                            metadata={"text": _words(rng, 10), "reference_table": [("<REF_3>", "o://shared")],
                                      "documents": second}),
            ReferenceHandle(id=3, token="<REF_3>", uri="o://r2", metadata=None)]
    rt = DeviceRuntime.for_planning(TinyPRAModel(_cfg()))
    tok = WordIdTokenizer(500, [f"<REF_{i}>" for i in range(1, 10)])
    _compare(rt, [{"references": refs}], tok)
