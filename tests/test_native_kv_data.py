"""Fixed-target native-KV stages and WikiText stages against the reference generators.

The reference's generators are the oracle: the same seeds must give the same
rows (every field of every file), for the synthetic lookup stage at several split
counts, for HotpotQA / QASPER probes built from small in-memory corpora, and for
the three WikiText layouts built from a generated local corpus (the reference's
corpus loader is pointed at the same rows).
"""

from __future__ import annotations

import importlib
import json
import random
import sys
from pathlib import Path

import pytest

from pdattention_b200.data import native_kv_benchmarks as nkv
from pdattention_b200.data.datasets import dataset_class_for_stage
from pdattention_b200.data.generators import wikitext as wt


def _read_stage(stage_dir: Path) -> dict:
    out = {}
    for name in ("documents", "references", "questions"):
        text = (stage_dir / f"{name}.jsonl").read_text(encoding="utf-8")
        out[name] = [json.loads(line) for line in text.splitlines() if line.strip()]
    manifest = stage_dir / "manifest.json"
    if manifest.exists():
        out["manifest"] = json.loads(manifest.read_text())
    return out


@pytest.fixture(scope="module")
def ref_nkv(ref):
    return importlib.import_module("data.native_kv_benchmarks")


def test_partition_bounds_cover_every_unit():
    for n, parts in ((63, 1), (63, 7), (63, 63), (1000, 255)):
        b = nkv.partition_bounds(n, parts)
        assert b[0] == 0 and b[-1] == n and all(hi > lo for lo, hi in zip(b, b[1:]))
    with pytest.raises(ValueError):
        nkv.partition_bounds(3, 4)


@pytest.mark.parametrize("split_count", [2, 8, 64])
def test_synthetic_stage_matches_reference(tmp_path, ref_nkv, split_count):
    ours = nkv.generate_synthetic_native_kv_dataset(tmp_path / "a", split_count=split_count, max_examples=24, seed=5)
    theirs = ref_nkv.generate_synthetic_native_kv_dataset(tmp_path / "b", split_count=split_count, max_examples=24,
                                                          seed=5)
    assert _read_stage(ours) == _read_stage(theirs)


def test_split_count_changes_only_the_partition(tmp_path):
    a = _read_stage(nkv.generate_synthetic_native_kv_dataset(tmp_path / "a", split_count=3, max_examples=6))
    b = _read_stage(nkv.generate_synthetic_native_kv_dataset(tmp_path / "b", split_count=32, max_examples=6))
    for qa, qb in zip(a["questions"], b["questions"]):
        assert qa["fixed_target_id"] == qb["fixed_target_id"]
        assert (qa["prompt"], qa["answer"], qa["source_text"]) == (qb["prompt"], qb["answer"], qb["source_text"])
    assert len(b["references"]) == 6 * 31
    with pytest.raises(ValueError):
        nkv.generate_synthetic_native_kv_dataset(tmp_path / "c", split_count=7)


def _hotpot_rows(n: int, seed: int = 0) -> list[dict]:
    rng = random.Random(seed)
    rows = []
    for i in range(n):
        titles = [f"T{i}_{j}" for j in range(4)]
        sentences = [[" ".join(f"w{rng.randrange(500)}" for _ in range(rng.randint(5, 12)))
                      for _ in range(rng.randint(2, 5))] for _ in titles]
        support_t = [titles[0], titles[2]]
        rows.append({"id": f"h{i}", "question": f"question {i}?", "answer": ["yes", "no", "Paris"][i % 3],
                     "type": "comparison", "level": "easy",
                     "context": {"title": titles, "sentences": sentences},
                     "supporting_facts": {"title": support_t, "sent_id": [0, 1]}})
    return rows


def test_hotpotqa_probes_match_reference(ref_nkv):
    rows = _hotpot_rows(60)
    ours = nkv.hotpotqa_answer_code_examples(rows, max_examples=20, seed=3)
    theirs = ref_nkv.hotpotqa_native_kv_examples(rows, max_examples=20, seed=3)
    assert [(e.id, e.answer, e.source_units, e.metadata) for e in ours] == \
        [(e.id, e.answer, tuple(nkv.EvidenceUnit(u.text, u.is_evidence) for u in e.source_units), e.metadata)
         for e in theirs]
    assert ours and {e.answer for e in ours} == {"yes", "no"}


def test_hotpotqa_official_json_layout(tmp_path):
    official = [{"_id": "x1", "question": "q?", "answer": "yes",
                 "context": [["A", ["a b c", "d e"]], ["B", ["f g"]]], "supporting_facts": [["A", 1]]}]
    path = tmp_path / "hotpot.json"
    path.write_text(json.dumps(official))
    rows = nkv.load_hotpotqa_rows("validation", path=path)
    assert rows[0]["id"] == "x1" and rows[0]["context"]["title"] == ["A", "B"]
    assert rows[0]["supporting_facts"] == {"title": ["A"], "sent_id": [1]}


def _qasper_papers(n: int, seed: int = 0) -> dict:
    rng = random.Random(seed)
    papers = {}
    for p in range(n):
        qas = []
        for q in range(3):
            votes = [{"answer": {"yes_no": rng.random() < 0.5,
                                 "evidence": [" ".join(f"e{rng.randrange(99)}" for _ in range(rng.randint(3, 9)))]}}
                     for _ in range(rng.randint(1, 3))]
            qas.append({"question_id": f"p{p}q{q}", "question": f"q{q}?", "answers": votes})
        papers[f"paper{p}"] = {"title": f"P{p}", "abstract": " ".join(f"a{rng.randrange(999)}" for _ in range(40)),
                               "full_text": [{"paragraphs": [" ".join(f"b{rng.randrange(999)}" for _ in range(30))]}],
                               "qas": qas}
    return papers


def test_qasper_probes_match_reference(ref_nkv):
    papers = _qasper_papers(12)
    ours = nkv.qasper_answer_code_examples(papers, max_examples=16, seed=9)
    theirs = ref_nkv.qasper_native_kv_examples(papers, max_examples=16, seed=9)
    assert [(e.id, e.answer, [u.text for u in e.source_units], e.metadata) for e in ours] == \
        [(e.id, e.answer, [u.text for u in e.source_units], e.metadata) for e in theirs]
    assert len(ours) > 0


def test_qasper_reads_a_local_split_file(tmp_path):
    path = tmp_path / "qasper-dev-v0.3.json"
    path.write_text(json.dumps(_qasper_papers(2)))
    assert set(nkv.load_qasper_papers("validation", path=path)) == {"paper0", "paper1"}
    with pytest.raises(FileNotFoundError):
        nkv.load_qasper_papers("train", cache_dir=tmp_path / "missing")


def _corpus(tmp_path: Path, paragraphs: int = 40) -> Path:
    rng = random.Random(11)
    lines = [""]
    for p in range(paragraphs):
        lines += [f" = Heading {p} = ", ""]
        lines.append(" ".join(f"tok{rng.randrange(3000)}" for _ in range(rng.randint(60, 260))))
        lines.append("")
    path = tmp_path / "wiki.train.raw"
    path.write_text("\n".join(lines), encoding="utf-8")
    return path


@pytest.fixture
def ref_datasets(ref, monkeypatch, tmp_path):
    mod = importlib.import_module("data.datasets")
    corpus = _corpus(tmp_path)
    rows = [{"text": line} for line in corpus.read_text(encoding="utf-8").splitlines()]
    monkeypatch.setattr(mod, "load_wikitext_splits", lambda *a, **k: {"train": rows})
    return mod, corpus


@pytest.mark.parametrize("kind", ["v1", "v2", "native"])
def test_wikitext_stages_match_reference(tmp_path, ref_datasets, kind):
    mod, corpus = ref_datasets
    if kind == "v1":
        ours = wt.generate_wikitext_reference_dataset(tmp_path / "a", corpus_path=corpus, max_examples=12,
                                                      min_words=70)
        theirs = mod.generate_wikitext_reference_dataset(tmp_path / "b", max_examples=12, min_words=70)
    elif kind == "v2":
        ours = wt.generate_wikitext_reference_dataset_v2(tmp_path / "a", corpus_path=corpus.parent,
                                                         max_examples=12, split_count=4)
        theirs = mod.generate_wikitext_reference_dataset_v2(tmp_path / "b", max_examples=12, split_count=4)
    else:
        ours = wt.generate_wikitext_nativekv_fixed_target_dataset(tmp_path / "a", split_count=8, corpus_path=corpus,
                                                                  max_examples=12)
        theirs = mod.generate_wikitext_nativekv_fixed_target_dataset(tmp_path / "b", split_count=8, max_examples=12)
    mine, oracle = _read_stage(ours), _read_stage(theirs)
    assert mine == oracle and len(mine["questions"]) > 0


def test_registry_generates_and_loads_the_stages(tmp_path):
    cls = dataset_class_for_stage("synthetic_nativekv_fixed_target")
    cls.generate(None, tmp_path, split_count=5, max_examples=4)
    ds = cls(tmp_path)
    assert len(ds) == 4 and len(ds[0].references) == 4 and ds[0].target_reference_ids == [1]
    cls = dataset_class_for_stage("wikitext2_references_v2")
    cls.generate(None, tmp_path, corpus_path=_corpus(tmp_path), max_examples=5)
    assert len(cls(tmp_path)) == 5


def test_wikitext_without_a_corpus_says_what_is_missing(tmp_path, monkeypatch):
    monkeypatch.setitem(sys.modules, "datasets", None)
    with pytest.raises(RuntimeError, match="corpus_path"):
        wt.generate_wikitext_reference_dataset(tmp_path)
