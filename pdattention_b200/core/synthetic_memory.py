"""Random flat memory-QA smoke examples (``src/pra_core/synthetic_memory.py``)."""

import random

from .datasets import DatasetExample
from .references import ReferenceTable

_COLOURS = ("red", "blue", "green", "yellow", "purple")
_ANIMALS = ("otter", "falcon", "tiger", "whale", "lynx")


def make_synthetic_examples(n: int = 100) -> list[DatasetExample]:
    examples = []
    for i in range(n):
        code = f"{random.choice(_COLOURS)}-{random.choice(_ANIMALS)}-{i}"
        uri = f"mem://doc{i}#summary"
        body = (f"Document {i}. This document contains project notes. The secret code is {code}. "
                f"The owner is team alpha. The rest of the document is filler text about systems and memory.")
        summary = f"Document {i} summary: contains a secret code and project notes."
        table = ReferenceTable()
        handle = table.register(uri, summary=summary)
        examples.append(DatasetExample(
            id=f"synthetic_{i}", prompt=f"Question: what is the secret code in {handle.token}? Answer:",
            target=f" {code}\n", refs={uri: body}, summaries={uri: summary}, reference_table=table,
            expected_ref_ids=[handle.id],
        ))
    return examples
