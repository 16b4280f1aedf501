"""Framework-neutral example loading from a stage folder.

A stage is a folder with three JSONL tables: ``documents.jsonl`` (``uri``,
``text``, optional ``summary``), ``references.jsonl`` (``uri``, optional ``id``,
``token``, ``summary``, ``metadata``) and ``questions.jsonl`` (``prompt``,
``answer``, optional ``id``, ``expected_ref_ids``, ``expected_anchors``).  Every
example gets its own ``ReferenceTable`` over all references of the stage, the
document text and summary of each handle, and the answer as the target
``" {answer}\\n"``.  Public names and results follow ``src/pra_core/datasets.py:9-103``.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from .references import ReferenceTable

_TABLES = ("documents", "references", "questions")


@dataclass
class DatasetExample:
    id: str
    prompt: str
    target: str
    refs: dict[str, str]
    summaries: dict[str, str]
    reference_table: ReferenceTable
    expected_ref_ids: list[int] = field(default_factory=list)
    expected_anchors: list[str] = field(default_factory=list)
    metadata: dict[str, Any] = field(default_factory=dict)


def load_jsonl(path) -> list[dict[str, Any]]:
    """Rows of a JSONL file (blank lines skipped); an absent file reads as no rows."""
    path = Path(path)
    if not path.exists():
        return []
    return [json.loads(line) for line in path.read_text(encoding="utf-8").splitlines() if line.strip()]


def _table(stage_path, name: str) -> list[dict[str, Any]]:
    return load_jsonl(Path(stage_path) / f"{name}.jsonl")


def load_documents(stage_path) -> list[dict[str, Any]]:
    return _table(stage_path, "documents")


def load_references(stage_path) -> list[dict[str, Any]]:
    return _table(stage_path, "references")


def load_questions(stage_path) -> list[dict[str, Any]]:
    return _table(stage_path, "questions")


def reference_table_from_rows(rows: list[dict[str, Any]]) -> ReferenceTable:
    """A table registering every reference row in order (explicit ids and tokens kept)."""
    table = ReferenceTable()
    for row in rows:
        table.register(uri=row["uri"], summary=row.get("summary"), metadata=row.get("metadata") or {},
                       id=row.get("id"), token=row.get("token"))
    return table


class _ExampleFactory:
    """Turns question rows into examples against one stage's documents and references."""

    def __init__(self, documents, references):
        self.text = {row["uri"]: row.get("text", "") for row in documents}
        self.summary = {row["uri"]: row.get("summary", "") for row in documents}
        self.references = references
        self.global_table = reference_table_from_rows(references)

    def __call__(self, question: dict, position: int) -> DatasetExample:
        table = reference_table_from_rows(self.references)
        handles = table.all()
        return DatasetExample(
            id=str(question.get("id", position)), prompt=question["prompt"], target=f" {question['answer']}\n",
            refs={h.uri: self.text.get(h.uri, "") for h in handles},
            summaries={h.uri: h.summary or self.summary.get(h.uri, "") for h in handles},
            reference_table=table, expected_ref_ids=list(map(int, question.get("expected_ref_ids", []))),
            expected_anchors=list(question.get("expected_anchors", [])),
            metadata={"question": question, "global_reference_table": self.global_table})


def build_examples(documents, references, questions, max_examples: int | None = None) -> list[DatasetExample]:
    make = _ExampleFactory(documents, references)
    return [make(question, i) for i, question in enumerate(questions[:max_examples])]


def load_dataset(stage: str, data_dir="data", max_examples: int | None = None) -> list[DatasetExample]:
    stage_path = Path(data_dir) / stage
    if not stage_path.exists():
        raise FileNotFoundError(f"Dataset stage not found: {stage_path}")
    documents, references, questions = (_table(stage_path, name) for name in _TABLES)
    return build_examples(documents, references, questions, max_examples)
