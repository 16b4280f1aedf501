"""Stage datasets over ``documents.jsonl`` / ``references.jsonl`` / ``questions.jsonl``.

Same stage registry and sample construction as ``src/data/datasets.py:27-306``:
a question row may restrict its references by ``reference_uris`` or
``reference_ids``; referenced documents with a ``reference_table`` carry the
whole document map so recursive resolution can find children.  The stage
generators here are this framework's own (``generators/``,
``native_kv_benchmarks``); WikiText, HotpotQA and QASPER stages read local
copies of those corpora (no downloads).
"""

from __future__ import annotations

import json
from abc import ABC, abstractmethod
from pathlib import Path
from typing import Any

from torch.utils.data import Dataset

from ..core.references import ReferenceTable
from .schemas import DatasetMetadata, QuestionSample, ReferenceSample


def read_jsonl(path: Path) -> list[dict[str, Any]]:
    path = Path(path)
    if not path.exists():
        return []
    with path.open("r", encoding="utf-8") as stream:
        return [json.loads(line) for line in stream if line.strip()]


def write_jsonl(path: str | Path, rows) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w", encoding="utf-8") as stream:
        for row in rows:
            stream.write(json.dumps(row) + "\n")
    return path


class PRADataset(Dataset, ABC):
    """A stage directory materialised as ``QuestionSample`` objects."""

    dataset_name = "pra"
    stage = "unknown"

    def __init__(self, data_dir: str | Path = "data", max_examples: int | None = None):
        self.data_dir = Path(data_dir)
        self.stage_path = self.data_dir / self.stage
        self.max_examples = max_examples
        self.metadata = DatasetMetadata(dataset_name=self.dataset_name, stage=self.stage)
        self.documents: list[dict] = []
        self.reference_rows: list[dict] = []
        self.question_rows: list[dict] = []
        self.samples: list[QuestionSample] = []
        self.load()

    def __len__(self) -> int:
        return len(self.samples)

    def __getitem__(self, idx: int) -> QuestionSample:
        return self.samples[idx]

    def load(self) -> None:
        self.documents = read_jsonl(self.stage_path / "documents.jsonl")
        self.reference_rows = read_jsonl(self.stage_path / "references.jsonl")
        self.question_rows = read_jsonl(self.stage_path / "questions.jsonl")
        if self.max_examples is not None:
            self.question_rows = self.question_rows[: self.max_examples]
        self.samples = self._build_samples()

    def build_reference_table(self, sample: QuestionSample | None = None) -> ReferenceTable:
        table = ReferenceTable()
        for ref in (sample.references if sample is not None else self._reference_samples()):
            table.register(uri=ref.uri, summary=ref.summary, metadata=ref.metadata, id=ref.id,
                           token=f"<REF_{ref.id}>")
        return table

    def evaluate(self, predictions: list[str]) -> dict[str, float]:
        hits = sum(s.answer.strip() in p for s, p in zip(self.samples, predictions))
        return {"answer_accuracy": hits / max(len(self.samples), 1)}

    @abstractmethod
    def generate(self, *args, **kwargs) -> None:
        raise NotImplementedError

    def _document_map(self, docs_by_uri: dict) -> dict:
        return {
            uri: {"text": d.get("text", ""), "summary": d.get("summary"),
                  "reference_table": d.get("reference_table", {}), "metadata": d.get("metadata", {}),
                  "version": d.get("version")}
            for uri, d in docs_by_uri.items()
        }

    def _reference_samples(self) -> list[ReferenceSample]:
        docs_by_uri = {row["uri"]: row for row in self.documents}
        shared_map = None
        out = []
        for row in self.reference_rows:
            doc = docs_by_uri.get(row["uri"], {})
            meta = dict(row.get("metadata") or {})
            meta.setdefault("text", doc.get("text", ""))
            meta.setdefault("title", doc.get("title"))
            meta.setdefault("anchors", doc.get("anchors", []))
            meta.setdefault("reference_table", dict(doc.get("reference_table") or {}))
            if meta["reference_table"]:
                if shared_map is None:
                    shared_map = self._document_map(docs_by_uri)
                meta.setdefault("documents", shared_map)
            out.append(ReferenceSample(id=int(row["id"]), uri=row["uri"], summary=row.get("summary") or doc.get("summary"),
                                       anchor=row.get("anchor"), metadata=meta))
        return out

    def _build_samples(self) -> list[QuestionSample]:
        refs = self._reference_samples()
        by_uri = {r.uri: r for r in refs}
        out = []
        for row in self.question_rows:
            uris = [str(u) for u in row.get("reference_uris") or []]
            ids = {int(i) for i in row.get("reference_ids") or []}
            chosen = refs
            if uris:
                chosen = [by_uri[u] for u in uris if u in by_uri]
            elif ids:
                chosen = [r for r in refs if r.id in ids]
            out.append(QuestionSample(
                id=str(row.get("id", len(out))), question=row["prompt"], answer=str(row["answer"]), references=chosen,
                target_reference_ids=[int(v) for v in row.get("expected_ref_ids", [])],
                target_reference_uris=[str(v) for v in row.get("expected_ref_uris", [])],
                target_chunk_ids=[str(v) for v in row.get("expected_chunk_ids", [])],
                target_chunk_spans=list(row.get("expected_chunk_spans", [])),
                metadata={"expected_anchors": list(row.get("expected_anchors", [])), "row": row,
                          "dataset": self.metadata},
            ))
        return out


def _stage_class(name: str, stage: str, generator: str, doc: str):
    def generate(self, *args, **kwargs):
        from . import generators

        return getattr(generators, generator)(*args, **kwargs)

    return type(name, (PRADataset,), {"dataset_name": name, "stage": stage, "generate": generate, "__doc__": doc,
                                      "generator_name": generator})


SyntheticMemoryQADataset = _stage_class("SyntheticMemoryQADataset", "stage0_synthetic_memory", "generate_synthetic",
                                        "Flat key:value memory QA.")
HierarchicalReferenceDataset = _stage_class("HierarchicalReferenceDataset", "stage1_hierarchical_synthetic",
                                            "generate_hierarchy", "Recursive child-first reference tables.")
CodeRepositoryDataset = _stage_class("CodeRepositoryDataset", "stage2_code_repos", "generate_code_repo",
                                     "Source files as references.")
WikipediaDataset = _stage_class("WikipediaDataset", "stage3_wikipedia", "generate_wikipedia", "Encyclopedia pages.")
BooksDataset = _stage_class("BooksDataset", "stage4_books", "generate_books", "Book chapters.")
DocumentationDataset = _stage_class("DocumentationDataset", "stage5_technical_docs", "generate_docs",
                                    "Technical documentation sections.")
GitHubRepositoryDataset = _stage_class("GitHubRepositoryDataset", "stage6_github_repos", "generate_code_repo",
                                       "Repository files.")
WikiTextReferenceDataset = _stage_class("WikiTextReferenceDataset", "wikitext2_references",
                                        "generate_wikitext_reference_dataset", "WikiText parts as references.")
WikiTextReferenceV2Dataset = _stage_class("WikiTextReferenceV2Dataset", "wikitext2_references_v2",
                                          "generate_wikitext_reference_dataset_v2", "Selection-labelled WikiText parts.")
WikiTextNativeKVFixedTargetDataset = _stage_class("WikiTextNativeKVFixedTargetDataset",
                                                  "wikitext2_nativekv_fixed_target",
                                                  "generate_wikitext_nativekv_fixed_target_dataset",
                                                  "WikiText history with a fixed tail and target.")
SyntheticNativeKVFixedTargetDataset = _stage_class("SyntheticNativeKVFixedTargetDataset",
                                                   "synthetic_nativekv_fixed_target",
                                                   "generate_synthetic_native_kv_dataset",
                                                   "Key/value retrieval with invariant target.")
HotpotQANativeKVFixedTargetDataset = _stage_class("HotpotQANativeKVFixedTargetDataset",
                                                  "hotpotqa_nativekv_fixed_target",
                                                  "generate_hotpotqa_native_kv_dataset",
                                                  "Balanced HotpotQA yes/no evidence (local corpus file).")
QASPERNativeKVFixedTargetDataset = _stage_class("QASPERNativeKVFixedTargetDataset", "qasper_nativekv_fixed_target",
                                                "generate_qasper_native_kv_dataset",
                                                "QASPER evidence spans (local corpus archive).")
# Synthetic benchmark stages of this framework.
KeyValueQADataset = _stage_class("KeyValueQADataset", "synthetic_kv_qa", "generate_kv_qa",
                                 "Seeded uniform-random documents with embedded key:value pairs.")
HierarchicalTokenDataset = _stage_class("HierarchicalTokenDataset", "synthetic_hierarchical_tokens",
                                        "generate_hierarchical_tokens",
                                        "Seeded depth-2 child-first reference trees of random tokens.")

DATASET_REGISTRY = {cls.stage: cls for cls in (
    SyntheticMemoryQADataset, HierarchicalReferenceDataset, CodeRepositoryDataset, DocumentationDataset,
    WikipediaDataset, BooksDataset, GitHubRepositoryDataset, WikiTextReferenceDataset, WikiTextReferenceV2Dataset,
    WikiTextNativeKVFixedTargetDataset, SyntheticNativeKVFixedTargetDataset, HotpotQANativeKVFixedTargetDataset,
    QASPERNativeKVFixedTargetDataset, KeyValueQADataset, HierarchicalTokenDataset,
)}


def dataset_class_for_stage(stage: str):
    try:
        return DATASET_REGISTRY[stage]
    except KeyError:
        raise KeyError(f"Unknown dataset stage: {stage}") from None


def load_wikitext_splits(dataset_name: str = "wikitext-2-raw-v1", *, cache_dir=None, corpus_path=None):
    """``{"train", "validation", "test"}`` rows of WikiText-2/103: from ``corpus_path`` (a
    directory with the raw ``wiki.{train,valid,test}.raw`` files) or from the ``datasets``
    package's cache.  Nothing is downloaded by this framework."""
    if dataset_name not in {"wikitext-2-raw-v1", "wikitext-103-raw-v1"}:
        raise ValueError(f"Unsupported WikiText dataset: {dataset_name}")
    if corpus_path is not None:
        root = Path(corpus_path)
        names = {"train": "wiki.train.raw", "validation": "wiki.valid.raw", "test": "wiki.test.raw"}
        return {split: [{"text": line} for line in (root / name).read_text(encoding="utf-8").splitlines()]
                for split, name in names.items()}
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise RuntimeError("WikiText needs corpus_path= (local wiki.*.raw files) or the 'datasets' package "
                           "with a cached copy") from exc
    return load_dataset("Salesforce/wikitext", dataset_name, cache_dir=str(cache_dir) if cache_dir else None)


def wikitext_documents(split, *, max_documents: int | None = None) -> list[str]:
    docs = [str(r["text"]).strip() for r in split if str(r["text"]).strip()]
    return docs[:max_documents] if max_documents is not None else docs
