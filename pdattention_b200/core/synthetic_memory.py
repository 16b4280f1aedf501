"""Flat memory-QA smoke examples: one referenced note per example holding a code word.

Each example's prompt asks for the code stored in its single reference; the
reference's full text states the code among filler sentences and its summary
only says that a code exists, so answering needs the memory, not the summary.
Draws use the module-level ``random`` state (seed it for repeatable sets).
"""

import random

from .datasets import DatasetExample
from .references import ReferenceTable

_ADJECTIVES = ("amber", "cobalt", "jade", "scarlet", "violet", "silver")
_NOUNS = ("heron", "badger", "comet", "maple", "harbor", "glacier")


def make_synthetic_examples(n: int = 100) -> list[DatasetExample]:
    examples = []
    for i in range(n):
        code = "-".join((random.choice(_ADJECTIVES), random.choice(_NOUNS), str(i)))
        uri = f"mem://doc{i}#summary"
        table = ReferenceTable()
        handle = table.register(uri, summary=f"Note {i}: records an access code among general notes.")
        text = (f"Note {i}. General notes about storage and scheduling follow. "
                f"Access code: {code}. Maintained by the platform group. "
                f"Further paragraphs discuss caches, queues and retries.")
        examples.append(DatasetExample(
            id=f"synthetic_{i}", prompt=f"Question: what is the access code in {handle.token}? Answer:",
            target=f" {code}\n", refs={uri: text}, summaries={uri: handle.summary}, reference_table=table,
            expected_ref_ids=[handle.id]))
    return examples
