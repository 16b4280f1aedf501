"""Seeded depth-2 child-first reference trees over a word-id vocabulary.

Every example owns ``roots`` root references.  Each root names ``children``
child documents and each child names ``grandchildren`` leaves through its
document ``reference_table``; with the defaults (2 roots, 1 child, 6 leaves)
an example resolves 16 references.  Documents are ``doc_tokens`` uniform-random
ids rendered as ``t<id>`` words so the text-based dataset format can carry a
large vocabulary through ``WordIdTokenizer``.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from pathlib import Path

from ..datasets import write_jsonl


@dataclass(frozen=True)
class HierarchicalTokenSpec:
    examples: int = 64
    roots: int = 2
    children: int = 1
    grandchildren: int = 6
    doc_tokens: int = 128
    prompt_tokens: int = 767
    vocab: int = 50257
    seed: int = 0

    @property
    def references_per_example(self) -> int:
        return self.roots * (1 + self.children * (1 + self.grandchildren))


def _words(rng: random.Random, count: int, vocab: int) -> list[str]:
    return [f"t{rng.randrange(1, vocab)}" for _ in range(count)]


def generate_hierarchical_tokens(out_dir, spec: HierarchicalTokenSpec | None = None, **overrides) -> Path:
    spec = spec or HierarchicalTokenSpec(**overrides)
    rng = random.Random(spec.seed)
    documents, references, questions = [], [], []

    def document(uri: str, child_uris: list[str]) -> None:
        table = {f"<REF_{i + 1}>": c for i, c in enumerate(child_uris)}
        handles = [f"<REF_{i + 1}>" for i in range(len(child_uris))]
        body = _words(rng, spec.doc_tokens - len(handles), spec.vocab)
        documents.append({"id": uri, "uri": uri, "text": " ".join(handles + body), "reference_table": table})

    for example in range(spec.examples):
        root_ids = []
        for r in range(spec.roots):
            root = f"tree://e{example}/r{r}"
            child_uris = []
            for c in range(spec.children):
                child = f"{root}/c{c}"
                leaves = [f"{child}/g{g}" for g in range(spec.grandchildren)]
                for leaf in leaves:
                    document(leaf, [])
                document(child, leaves)
                child_uris.append(child)
            document(root, child_uris)
            ref_id = len(references) + 1
            references.append({"id": ref_id, "token": f"<REF_{ref_id}>", "uri": root})
            root_ids.append((ref_id, root))
        handles = [f"<REF_{ref_id}>" for ref_id, _ in root_ids]
        filler = _words(rng, spec.prompt_tokens - len(handles), spec.vocab)
        answer = f"t{rng.randrange(1, spec.vocab)}"
        questions.append({"id": f"tree-{example}", "prompt": " ".join(handles + filler), "answer": answer,
                          "reference_uris": [u for _, u in root_ids],
                          "expected_ref_ids": [root_ids[0][0]]})
    out = Path(out_dir)
    write_jsonl(out / "documents.jsonl", documents)
    write_jsonl(out / "references.jsonl", references)
    write_jsonl(out / "questions.jsonl", questions)
    return out
