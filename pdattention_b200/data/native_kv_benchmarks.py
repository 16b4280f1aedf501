"""Fixed-target native-KV benchmark stages (transport / routing isolation).

A benchmark example is an ordered list of *source units* (words or facts, some
marked as evidence), a short question and its answer.  A stage written at split
count ``S`` turns the source into ``S - 1`` references by cutting the unit list at
``floor(i * n / (S - 1))``; everything else (source text, question, answer,
example order) is identical across split counts, so a loss difference between
two partitions measures memory partitioning and nothing else
(``src/data/native_kv_benchmarks.py:1-6``).

The writers here produce the reference's stage layout (``documents.jsonl`` /
``references.jsonl`` / ``questions.jsonl`` + ``manifest.json``, the same field
names and the same ``benchmark://`` URIs), which the dataset classes and the
reference's loaders read.  Three example sources:

* ``synthetic_fixed_position_examples``: 63 one-bit key/value facts per
  example, the queried fact at a fixed position; the draws follow the
  reference's seeded procedure so the stage is the same data
  (``src/data/native_kv_benchmarks.py:169-221``);
* ``hotpotqa_answer_code_examples`` / ``qasper_answer_code_examples``: yes/no
  questions turned into "return the answer code" probes over natural text.
  There is no network here, so the rows come from a local file (HotpotQA
  distractor-setting JSON / JSONL, QASPER's official archive or its JSON) or,
  for HotpotQA, from the ``datasets`` package when it is importable and the
  corpus is cached (``src/data/native_kv_benchmarks.py:224-506``).
"""

from __future__ import annotations

import hashlib
import json
import random
import string
import tarfile
from collections.abc import Callable, Iterable, Iterator, Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any


NATIVE_KV_SPLIT_COUNTS = (2, 3, 5, 8, 16, 32, 64)
NATIVE_KV_SCALE_SPLIT_COUNTS = (*NATIVE_KV_SPLIT_COUNTS, 128, 256)
ANSWER_CODE_QUESTION = " Question: Return the AnswerCode. Answer:"
QASPER_SPLIT_FILES = {"train": "qasper-train-v0.3.json", "validation": "qasper-dev-v0.3.json"}


@dataclass(frozen=True)
class EvidenceUnit:
    """One indivisible source unit; ``is_evidence`` marks units that support the answer."""

    text: str
    is_evidence: bool = False


@dataclass(frozen=True)
class NativeKVBenchmarkExample:
    """Source units, tail question and answer of one example (dataset neutral)."""

    id: str
    source_units: tuple[EvidenceUnit, ...]
    question: str
    answer: str
    metadata: dict = field(default_factory=dict)


def stable_digest(*parts: object) -> str:
    """sha256 hex of the parts joined by newlines (seeds and target ids that survive re-runs)."""
    return hashlib.sha256("\n".join(map(str, parts)).encode("utf-8")).hexdigest()


def partition_bounds(n_units: int, parts: int) -> list[int]:
    """Cut points ``floor(i * n / parts)`` for ``i = 0..parts``: ``parts`` non-empty ranges."""
    if parts < 1:
        raise ValueError("reference_count must be positive")
    if n_units < parts:
        raise ValueError(f"Need at least {parts} source units, received {n_units}")
    return [i * n_units // parts for i in range(parts + 1)]


def _stage_rows(example: NativeKVBenchmarkExample, dataset_name: str, split_count: int, version: str):
    """Documents, references and the question row of one example at ``split_count``."""
    units = example.source_units
    cuts = partition_bounds(len(units), split_count - 1)
    docs, refs, uris = [], [], []
    hits: list[tuple[int, str, int, int]] = []  # (reference id, uri, first unit, end unit)
    for ref_id, (lo, hi) in enumerate(zip(cuts[:-1], cuts[1:]), start=1):
        group = units[lo:hi]
        uri = f"benchmark://{dataset_name}/{example.id}/part-{ref_id}"
        evidence = any(u.is_evidence for u in group)
        if evidence:
            hits.append((ref_id, uri, lo, hi))
        uris.append(uri)
        docs.append({"id": f"{example.id}-part-{ref_id}", "uri": uri,
                     "title": f"{dataset_name} {example.id} part {ref_id}", "text": " ".join(u.text for u in group)})
        refs.append({"id": ref_id, "token": f"<REF_{ref_id}>", "uri": uri,
                     "metadata": {"dataset": dataset_name, "example_id": example.id, "unit_span": [lo, hi],
                                  "is_evidence": evidence, "split_count": split_count}})
    source_text = " ".join(u.text for u in units)
    question = {
        "id": example.id, "prompt": example.question, "answer": example.answer, "reference_uris": uris,
        "expected_ref_ids": [h[0] for h in hits], "expected_ref_uris": [h[1] for h in hits],
        "expected_chunk_spans": [{"reference_uri": h[1], "unit_start": h[2], "unit_end": h[3]} for h in hits],
        "source_text": source_text, "source_unit_count": len(units), "split_count": split_count,
        "reference_count": split_count - 1,
        "fixed_target_id": stable_digest(example.id, source_text, example.question, example.answer),
        "generation_version": version, **example.metadata,
    }
    return docs, refs, question


def write_native_kv_benchmark(data_dir, *, stage: str, dataset_name: str, split_count: int,
                              examples: Iterable[NativeKVBenchmarkExample], generation_version: str) -> Path:
    """Write one fixed-target partition of ``examples`` under ``data_dir/stage``."""
    if split_count not in NATIVE_KV_SCALE_SPLIT_COUNTS:
        raise ValueError("split_count must be one of " + ", ".join(map(str, NATIVE_KV_SCALE_SPLIT_COUNTS)))
    out = Path(data_dir) / stage
    documents, references, questions = [], [], []
    for example in examples:
        docs, refs, question = _stage_rows(example, dataset_name, split_count, generation_version)
        documents += docs
        references += refs
        questions.append(question)
    for name, rows in (("documents", documents), ("references", references), ("questions", questions)):
        _write_ascii_jsonl(out / f"{name}.jsonl", rows)
    manifest = {"dataset": dataset_name, "split_count": split_count, "example_count": len(questions),
                "generation_version": generation_version}
    (out / "manifest.json").write_text(json.dumps(manifest, indent=2), encoding="utf-8")
    return out


def _write_ascii_jsonl(path: Path, rows: list[dict]) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w", encoding="utf-8") as stream:
        stream.writelines(json.dumps(row, ensure_ascii=True) + "\n" for row in rows)


# ---------------------------------------------------------------------------
# Synthetic fixed-position key/value lookup
# ---------------------------------------------------------------------------

_TARGET_KEY = "@"
_KEY_ALPHABET = string.ascii_lowercase + string.ascii_uppercase + string.digits


def synthetic_fixed_position_examples(*, max_examples: int = 320, seed: int = 1729) -> list[NativeKVBenchmarkExample]:
    """63 one-bit facts ``<key><bit>`` per example; the queried key ``@`` is always first.

    Per example ``i`` a generator seeded ``seed + 104729 i`` shuffles the 62 other
    keys, draws the answer bit, then one bit per fact (the target's bit is the
    answer).  A model without memory can only guess (answer space 2); every
    example carries exact evidence labels."""
    out = []
    for i in range(max_examples):
        rng = random.Random(seed + i * 104_729)
        others = list(_KEY_ALPHABET)
        rng.shuffle(others)
        keys = [_TARGET_KEY, *others]
        answer = str(rng.randrange(2))
        bits = [str(rng.randrange(2)) for _ in keys]
        bits[0] = answer
        units = tuple(EvidenceUnit(k + b, is_evidence=(pos == 0)) for pos, (k, b) in enumerate(zip(keys, bits)))
        out.append(NativeKVBenchmarkExample(
            id=f"synthetic-native-{i:05d}", source_units=units, question="?", answer=answer,
            metadata={"task_type": "fixed_position_key_value_retrieval", "target_source_unit": 0,
                      "local_context_sufficient": False, "answer_space_size": 2}))
    return out


def generate_synthetic_native_kv_dataset(data_dir, *, split_count: int, max_examples: int = 320,
                                         seed: int = 1729) -> Path:
    """Write the synthetic fixed-position lookup stage (``synthetic_nativekv_fixed_target``)."""
    return write_native_kv_benchmark(data_dir, stage="synthetic_nativekv_fixed_target",
                                     dataset_name="synthetic_native_kv", split_count=split_count,
                                     examples=synthetic_fixed_position_examples(max_examples=max_examples, seed=seed),
                                     generation_version="synthetic_nativekv_fixed_target_v5")


# ---------------------------------------------------------------------------
# Answer-code probes over natural text (HotpotQA, QASPER)
# ---------------------------------------------------------------------------

@dataclass
class _Candidate:
    """A yes/no question with its evidence words and the pool distractors are drawn from."""

    example_id: str
    answer: str                      # "yes" | "no"
    evidence_words: list[str]
    distractor_pool: list[str]
    seed_material: tuple
    metadata: dict


def _answer_code_example(c: _Candidate, seed: int, units_total: int) -> NativeKVBenchmarkExample | None:
    """``[AnswerCode, <answer>]`` (the evidence anchor), the evidence words, then distractor
    words sampled without replacement from the pool and kept in pool order; ``None`` when the
    pool cannot fill the budget."""
    needed = units_total - len(c.evidence_words) - 2
    if needed < 0 or len(c.distractor_pool) < needed:
        return None
    rng = random.Random(int(stable_digest(seed, *c.seed_material)[:16], 16))
    picks = sorted(rng.sample(range(len(c.distractor_pool)), needed))
    units = [EvidenceUnit("AnswerCode", True), EvidenceUnit(c.answer, True)]
    units += [EvidenceUnit(w) for w in c.evidence_words]
    units += [EvidenceUnit(c.distractor_pool[j]) for j in picks]
    meta = dict(c.metadata)
    meta.update(evidence_unit_count=len(c.evidence_words), local_context_sufficient=False, answer_space_size=2)
    return NativeKVBenchmarkExample(id=c.example_id, source_units=tuple(units), question=ANSWER_CODE_QUESTION,
                                    answer=c.answer, metadata=meta)


def _balanced(examples: Iterable[NativeKVBenchmarkExample], max_examples: int, seed: int):
    """Equal numbers of "yes" and "no" examples (each label shuffled with its own seed), then
    the union shuffled."""
    by_label: dict[str, list] = {"yes": [], "no": []}
    for ex in examples:
        by_label[ex.answer].append(ex)
    per_label = min(len(by_label["yes"]), len(by_label["no"]), max_examples // 2)
    picked = []
    for offset, label in enumerate(("yes", "no")):
        pool = by_label[label]
        random.Random(seed + offset * 1_000_003).shuffle(pool)
        picked += pool[:per_label]
    random.Random(seed + 2_000_003).shuffle(picked)
    return picked[:max_examples]


def _probe_examples(candidates: Iterator[_Candidate], *, max_examples: int, seed: int, source_unit_count: int,
                    max_evidence_units: int, trim_evidence: bool) -> list[NativeKVBenchmarkExample]:
    built = []
    for c in candidates:
        if trim_evidence:
            c.evidence_words = c.evidence_words[:max_evidence_units]
        if not c.evidence_words or len(c.evidence_words) > max_evidence_units:
            continue
        ex = _answer_code_example(c, seed, source_unit_count)
        if ex is not None:
            built.append(ex)
    return _balanced(built, max_examples, seed)


def _hotpot_candidates(rows: Iterable[dict[str, Any]]) -> Iterator[_Candidate]:
    for row in rows:
        answer = str(row.get("answer", "")).strip().lower()
        if answer not in ("yes", "no"):
            continue
        facts = row["supporting_facts"]
        support = {(str(t), int(s)) for t, s in zip(facts["title"], facts["sent_id"])}
        evidence, pool, sentences = [], [], []
        ctx = row["context"]
        for title, paragraph in zip(ctx["title"], ctx["sentences"]):
            for sid, sentence in enumerate(paragraph):
                text = str(sentence).strip()
                if (str(title), sid) in support:
                    evidence += text.split()
                    sentences.append(text)
                else:
                    pool += text.split()
        yield _Candidate(
            example_id=f"hotpotqa-{row['id']}", answer=answer, evidence_words=evidence, distractor_pool=pool,
            seed_material=(row.get("id", ""),),
            metadata={"task_type": "hotpotqa_answer_code_transport_probe",
                      "original_question": str(row["question"]).strip(), "source_dataset_id": str(row["id"]),
                      "hotpot_type": str(row.get("type", "")), "hotpot_level": str(row.get("level", "")),
                      "supporting_sentences": sentences})


def hotpotqa_answer_code_examples(rows: Iterable[dict[str, Any]], *, max_examples: int, seed: int,
                                  source_unit_count: int = 63, max_evidence_units: int = 59):
    """Balanced HotpotQA yes/no rows (distractor setting) as answer-code probes: the supporting
    sentences' words are the evidence, other context sentences supply distractors."""
    return _probe_examples(_hotpot_candidates(rows), max_examples=max_examples, seed=seed,
                           source_unit_count=source_unit_count, max_evidence_units=max_evidence_units,
                           trim_evidence=False)


def _qasper_candidates(papers: dict[str, dict[str, Any]]) -> Iterator[_Candidate]:
    seen = {"yes": 0, "no": 0}  # fallback question ids (v0.3 always carries ``question_id``)
    for paper_id, paper in papers.items():
        words = str(paper.get("abstract", "")).split()
        for section in paper.get("full_text", []):
            for paragraph in section.get("paragraphs", []):
                words += str(paragraph).split()
        for qa in paper.get("qas", []):
            votes = [(bool(a["answer"]["yes_no"]), list(a["answer"].get("evidence") or []))
                     for a in qa.get("answers", []) if a.get("answer", {}).get("yes_no") is not None]
            if not votes:
                continue
            label = "yes" if 2 * sum(v for v, _ in votes) >= len(votes) else "no"
            agreeing = [t for v, ev in votes if ("yes" if v else "no") == label for t in ev if str(t).strip()]
            if not agreeing:
                continue
            shortest = min(agreeing, key=lambda t: len(t.split()))
            qid = str(qa.get("question_id", seen[label]))
            seen[label] += 1
            yield _Candidate(
                example_id=f"qasper-{paper_id}-{qid}", answer=label, evidence_words=shortest.split(),
                distractor_pool=words, seed_material=(paper_id, qid),
                metadata={"task_type": "qasper_answer_code_transport_probe", "paper_id": str(paper_id),
                          "paper_title": str(paper.get("title", "")), "question_id": qid,
                          "original_question": str(qa.get("question", "")), "supporting_evidence": agreeing})


def qasper_answer_code_examples(papers: dict[str, dict[str, Any]], *, max_examples: int, seed: int,
                                source_unit_count: int = 63, max_evidence_units: int = 59):
    """Balanced QASPER yes/no questions as answer-code probes: the shortest agreeing evidence
    span (trimmed to the evidence budget) is the evidence, the paper's words the distractors."""
    return _probe_examples(_qasper_candidates(papers), max_examples=max_examples, seed=seed,
                           source_unit_count=source_unit_count, max_evidence_units=max_evidence_units,
                           trim_evidence=True)


# ---------------------------------------------------------------------------
# Local corpus loaders (no network on this framework's hosts)
# ---------------------------------------------------------------------------

def load_hotpotqa_rows(dataset_split: str, *, path: str | Path | None = None, cache_dir=None) -> list[dict]:
    """HotpotQA distractor-setting rows: from ``path`` (the official JSON list, or JSONL in the
    Hugging Face row layout), else from the ``datasets`` package's cache."""
    if path is not None:
        return [_hotpot_hf_layout(r) for r in _read_json_rows(Path(path))]
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise RuntimeError("HotpotQA needs a local file (path=...) or the 'datasets' package with a cached "
                           "copy of hotpotqa/hotpot_qa") from exc
    return list(load_dataset("hotpotqa/hotpot_qa", "distractor", split=dataset_split,
                             cache_dir=str(cache_dir) if cache_dir else None))


def _read_json_rows(path: Path) -> list[dict]:
    text = path.read_text(encoding="utf-8")
    stripped = text.lstrip()
    if stripped.startswith("["):
        return json.loads(text)
    return [json.loads(line) for line in text.splitlines() if line.strip()]


def _hotpot_hf_layout(row: dict) -> dict:
    """The official HotpotQA JSON (``_id``, ``context`` as [title, sentences] pairs,
    ``supporting_facts`` as [title, sent_id] pairs) in the Hugging Face column layout."""
    if isinstance(row.get("context"), dict):
        return row
    ctx = row.get("context", [])
    facts = row.get("supporting_facts", [])
    return {**row, "id": row.get("id", row.get("_id")),
            "context": {"title": [c[0] for c in ctx], "sentences": [c[1] for c in ctx]},
            "supporting_facts": {"title": [f[0] for f in facts], "sent_id": [f[1] for f in facts]}}


def load_qasper_papers(dataset_split: str, *, cache_dir: str | Path | None = None,
                       path: str | Path | None = None) -> dict[str, dict[str, Any]]:
    """QASPER v0.3 papers of ``dataset_split`` from ``path`` (the split's JSON or the official
    ``qasper-train-dev-v0.3.tgz``) or from that archive under ``cache_dir``."""
    if dataset_split not in QASPER_SPLIT_FILES:
        raise ValueError(f"Unsupported QASPER split: {dataset_split}")
    member = QASPER_SPLIT_FILES[dataset_split]
    source = Path(path) if path is not None else Path(cache_dir or Path.home() / ".cache" / "qasper") / \
        "qasper-train-dev-v0.3.tgz"
    if not source.exists():
        raise FileNotFoundError(f"QASPER needs {source} (the official v0.3 archive or {member}); this framework "
                                "does not download corpora")
    if source.suffix == ".json":
        return json.loads(source.read_text(encoding="utf-8"))
    with tarfile.open(source, "r:gz") as archive:
        handle = archive.extractfile(member)
        if handle is None:
            raise FileNotFoundError(member)
        return json.load(handle)


def _require_count(examples: Sequence, wanted: int, what: str):
    if len(examples) < wanted:
        raise ValueError(f"{what} yielded {len(examples)} usable balanced examples; requested {wanted}")
    return examples


def generate_hotpotqa_native_kv_dataset(data_dir, *, split_count: int, dataset_split: str, max_examples: int,
                                        seed: int, source_unit_count: int = 63, cache_dir=None,
                                        source_path: str | Path | None = None) -> Path:
    """Write the balanced HotpotQA answer-code stage (``hotpotqa_nativekv_fixed_target``)."""
    rows = load_hotpotqa_rows(dataset_split, path=source_path, cache_dir=cache_dir)
    examples = _require_count(hotpotqa_answer_code_examples(rows, max_examples=max_examples, seed=seed,
                                                            source_unit_count=source_unit_count),
                              max_examples, f"HotpotQA {dataset_split}")
    return write_native_kv_benchmark(data_dir, stage="hotpotqa_nativekv_fixed_target", dataset_name="hotpotqa",
                                     split_count=split_count, examples=examples,
                                     generation_version="hotpotqa_nativekv_answer_code_v3")


def generate_qasper_native_kv_dataset(data_dir, *, split_count: int, dataset_split: str, max_examples: int,
                                      seed: int, source_unit_count: int = 63, cache_dir=None,
                                      source_path: str | Path | None = None) -> Path:
    """Write the balanced QASPER answer-code stage (``qasper_nativekv_fixed_target``)."""
    papers = load_qasper_papers(dataset_split, cache_dir=cache_dir, path=source_path)
    examples = _require_count(qasper_answer_code_examples(papers, max_examples=max_examples, seed=seed,
                                                          source_unit_count=source_unit_count),
                              max_examples, f"QASPER {dataset_split}")
    return write_native_kv_benchmark(data_dir, stage="qasper_nativekv_fixed_target", dataset_name="qasper",
                                     split_count=split_count, examples=examples,
                                     generation_version="qasper_nativekv_answer_code_v2")


GENERATORS: dict[str, Callable[..., Path]] = {
    "synthetic_nativekv_fixed_target": generate_synthetic_native_kv_dataset,
    "hotpotqa_nativekv_fixed_target": generate_hotpotqa_native_kv_dataset,
    "qasper_nativekv_fixed_target": generate_qasper_native_kv_dataset,
}
