"""Non-tensor example records (``src/data/schemas.py:5-37``)."""

from dataclasses import dataclass, field
from typing import Any


@dataclass(frozen=True)
class ReferenceSample:
    id: int
    uri: str
    summary: str | None = None
    anchor: str | None = None
    metadata: dict[str, Any] = field(default_factory=dict)


@dataclass(frozen=True)
class QuestionSample:
    id: str
    question: str
    answer: str
    references: list[ReferenceSample]
    target_reference_ids: list[int] = field(default_factory=list)
    target_reference_uris: list[str] = field(default_factory=list)
    target_chunk_ids: list[str] = field(default_factory=list)
    target_chunk_spans: list[dict[str, Any]] = field(default_factory=list)
    metadata: dict[str, Any] = field(default_factory=dict)


@dataclass(frozen=True)
class DatasetMetadata:
    dataset_name: str
    stage: str
    version: str = "0.1.0"
