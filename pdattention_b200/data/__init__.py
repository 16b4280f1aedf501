"""Data layer: schemas, tokenizers, stage datasets, collator and data modules."""

from .collators import PRACollator
from .datamodules import PRADataModule
from .datasets import (
    DATASET_REGISTRY,
    BooksDataset,
    CodeRepositoryDataset,
    DocumentationDataset,
    GitHubRepositoryDataset,
    HierarchicalReferenceDataset,
    HierarchicalTokenDataset,
    KeyValueQADataset,
    PRADataset,
    SyntheticMemoryQADataset,
    WikipediaDataset,
    WikiTextNativeKVFixedTargetDataset,
    WikiTextReferenceDataset,
    dataset_class_for_stage,
    load_wikitext_splits,
    read_jsonl,
    wikitext_documents,
    write_jsonl,
)
from .language_modeling import TokenBlockDataset, WikiTextDataModule
from .schemas import DatasetMetadata, QuestionSample, ReferenceSample
from .tokenizer import BPETokenizer, PRATokenizer, WordIdTokenizer

__all__ = [name for name in dir() if not name.startswith("_")]
