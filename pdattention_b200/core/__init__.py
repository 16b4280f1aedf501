"""Framework-neutral reference core (no torch)."""

from .datasets import DatasetExample, load_dataset
from .references import ReferenceHandle, ReferenceTable, ResolvedReference

__all__ = ["DatasetExample", "ReferenceHandle", "ReferenceTable", "ResolvedReference", "load_dataset"]
