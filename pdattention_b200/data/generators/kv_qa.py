"""Seeded key:value memory QA (character tokenizer).

Each question carries 2-4 ``<REF_n>`` handles; each handle's document is
256-1024 characters drawn uniformly from a fixed alphabet with 8 embedded
``key:value`` pairs.  The question names one key; the answer is its value.
"""

from __future__ import annotations

import random
import string
from pathlib import Path

from ..datasets import write_jsonl

_FILLER = string.ascii_lowercase + string.digits + " "


def _token(rng: random.Random, prefix: str) -> str:
    return prefix + "".join(rng.choice(string.ascii_uppercase + string.digits) for _ in range(3))


def generate_kv_qa(out_dir, n: int = 64, seed: int = 0, min_refs: int = 2, max_refs: int = 4,
                   min_doc_tokens: int = 256, max_doc_tokens: int = 1024, pairs_per_doc: int = 8) -> Path:
    rng = random.Random(seed)
    out = Path(out_dir)
    documents, references, questions = [], [], []
    for example in range(n):
        ref_count = rng.randint(min_refs, max_refs)
        uris, pairs_by_uri = [], {}
        for local in range(ref_count):
            uri = f"kv://example{example}/doc{local}"
            length = rng.randint(min_doc_tokens, max_doc_tokens)
            pairs = [(_token(rng, "K"), _token(rng, "V")) for _ in range(pairs_per_doc)]
            body = [rng.choice(_FILLER) for _ in range(length)]
            insert_at = sorted(rng.sample(range(max(length - 10, 1)), pairs_per_doc))
            text = []
            cursor = 0
            for position, (key, value) in zip(insert_at, pairs):
                text.append("".join(body[cursor:position]))
                text.append(f" {key}:{value} ")
                cursor = position
            text.append("".join(body[cursor:]))
            documents.append({"id": f"e{example}d{local}", "uri": uri, "text": "".join(text)})
            ref_id = len(references) + 1
            references.append({"id": ref_id, "token": f"<REF_{ref_id}>", "uri": uri})
            uris.append((ref_id, uri))
            pairs_by_uri[uri] = pairs
        target_id, target_uri = rng.choice(uris)
        key, value = rng.choice(pairs_by_uri[target_uri])
        handles = " ".join(f"<REF_{ref_id}>" for ref_id, _ in uris)
        questions.append({"id": f"kvqa-{example}", "prompt": f"{handles} value of {key}?", "answer": value,
                          "reference_uris": [u for _, u in uris], "expected_ref_ids": [target_id]})
    write_jsonl(out / "documents.jsonl", documents)
    write_jsonl(out / "references.jsonl", references)
    write_jsonl(out / "questions.jsonl", questions)
    return out
