"""Framework-neutral example loading (``src/pra_core/datasets.py:9-103``)."""

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from .references import ReferenceTable


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


def load_jsonl(path: str | Path) -> list[dict[str, Any]]:
    path = Path(path)
    if not path.exists():
        return []
    with path.open("r", encoding="utf-8") as stream:
        return [json.loads(line) for line in stream if line.strip()]


def load_documents(stage_path: str | Path) -> list[dict[str, Any]]:
    return load_jsonl(Path(stage_path) / "documents.jsonl")


def load_references(stage_path: str | Path) -> list[dict[str, Any]]:
    return load_jsonl(Path(stage_path) / "references.jsonl")


def load_questions(stage_path: str | Path) -> list[dict[str, Any]]:
    return load_jsonl(Path(stage_path) / "questions.jsonl")


def reference_table_from_rows(rows: list[dict[str, Any]]) -> ReferenceTable:
    table = ReferenceTable()
    for row in rows:
        table.register(uri=row["uri"], summary=row.get("summary"), metadata=row.get("metadata") or {},
                       id=row.get("id"), token=row.get("token"))
    return table


def build_examples(documents, references, questions, max_examples: int | None = None) -> list[DatasetExample]:
    docs = {row["uri"]: row for row in documents}
    global_table = reference_table_from_rows(references)
    out = []
    for row in questions[:max_examples]:
        table = reference_table_from_rows(references)
        refs, summaries = {}, {}
        for handle in table.all():
            doc = docs.get(handle.uri) or {}
            refs[handle.uri] = doc.get("text", "")
            summaries[handle.uri] = handle.summary or doc.get("summary", "")
        out.append(DatasetExample(
            id=str(row.get("id", len(out))), prompt=row["prompt"], target=f" {row['answer']}\n",
            refs=refs, summaries=summaries, reference_table=table,
            expected_ref_ids=[int(v) for v in row.get("expected_ref_ids", [])],
            expected_anchors=list(row.get("expected_anchors", [])),
            metadata={"question": row, "global_reference_table": global_table},
        ))
    return out


def load_dataset(stage: str, data_dir: str | Path = "data", max_examples: int | None = None) -> list[DatasetExample]:
    stage_path = Path(data_dir) / stage
    if not stage_path.exists():
        raise FileNotFoundError(f"Dataset stage not found: {stage_path}")
    return build_examples(load_documents(stage_path), load_references(stage_path), load_questions(stage_path),
                          max_examples)
