"""Seeded stage generators.

``generate_kv_qa`` writes the flat key:value memory QA stage (2-4 ``<REF_n>`` per
question, documents of uniform-random tokens with 8 embedded key:value pairs).
``generate_hierarchical_tokens`` writes depth-2 child-first reference trees of
uniform-random token ids for the data-parallel training benchmark.  The small
demo stages (code, docs, books, wikipedia) are deterministic toy corpora.  The
WikiText stages read a local corpus (``wikitext``); the fixed-target native-KV
stages live in ``pdattention_b200.data.native_kv_benchmarks``.
"""

from .synthetic import (
    generate_books,
    generate_code_repo,
    generate_docs,
    generate_hierarchy,
    generate_synthetic,
    generate_wikipedia,
)
from .wikitext import (
    generate_wikitext_nativekv_fixed_target_dataset,
    generate_wikitext_reference_dataset,
    generate_wikitext_reference_dataset_v2,
)
from ..native_kv_benchmarks import (
    generate_hotpotqa_native_kv_dataset,
    generate_qasper_native_kv_dataset,
    generate_synthetic_native_kv_dataset,
)
from .kv_qa import generate_kv_qa
from .hierarchical_tokens import HierarchicalTokenSpec, generate_hierarchical_tokens

__all__ = [
    "HierarchicalTokenSpec",
    "generate_books",
    "generate_code_repo",
    "generate_docs",
    "generate_hierarchical_tokens",
    "generate_hierarchy",
    "generate_kv_qa",
    "generate_synthetic",
    "generate_hotpotqa_native_kv_dataset",
    "generate_qasper_native_kv_dataset",
    "generate_synthetic_native_kv_dataset",
    "generate_wikipedia",
    "generate_wikitext_nativekv_fixed_target_dataset",
    "generate_wikitext_reference_dataset",
    "generate_wikitext_reference_dataset_v2",
]
