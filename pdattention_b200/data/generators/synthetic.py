"""Small deterministic demo corpora for the named stages."""

from __future__ import annotations

import random
from pathlib import Path

from ..datasets import write_jsonl


def _write_stage(out_dir, documents, references, questions) -> Path:
    out = Path(out_dir)
    write_jsonl(out / "documents.jsonl", documents)
    write_jsonl(out / "references.jsonl", references)
    write_jsonl(out / "questions.jsonl", questions)
    return out


def _facts_stage(out_dir, n: int, kind: str, subjects: list[tuple[str, str]], seed: int):
    rng = random.Random(seed)
    documents, references, questions = [], [], []
    for index, (name, fact) in enumerate(subjects[:max(n, 2)], start=1):
        uri = f"memory://{kind}/{name}"
        code = f"CODE{rng.randint(10, 99)}"
        documents.append({"id": f"{kind}{index}", "uri": uri, "title": name,
                          "text": f"Title: {name}. {fact}. Secret code: {code}.", "summary": f"Facts about {name}."})
        references.append({"id": index, "token": f"<REF_{index}>", "uri": uri, "summary": f"Facts about {name}."})
        others = [r for r in range(1, len(subjects) + 1) if r != index][:2]
        tokens = " ".join(f"<REF_{i}>" for i in sorted([index, *others]))
        questions.append({"id": f"{kind}_q{index}", "prompt": f"What is the secret code for {name}? {tokens}",
                          "answer": code, "expected_ref_ids": [index]})
    return _write_stage(out_dir, documents, references, questions)


def generate_synthetic(out_dir, n: int = 4, seed: int = 0) -> Path:
    subjects = [("cat", "It hunts mice"), ("dog", "It guards houses"), ("owl", "It hunts at night"),
                ("bee", "It makes honey"), ("fox", "It is clever"), ("elk", "It has antlers")]
    return _facts_stage(out_dir, n, "animal", subjects, seed)


def generate_code_repo(out_dir, n: int = 3, seed: int = 0) -> Path:
    subjects = [("auth.py", "Defines login()"), ("db.py", "Defines connect()"), ("api.py", "Defines route()")]
    return _facts_stage(out_dir, n, "repo", subjects, seed)


def generate_docs(out_dir, n: int = 3, seed: int = 0) -> Path:
    subjects = [("install", "Run pip install"), ("config", "Edit config.yml"), ("deploy", "Use the deploy script")]
    return _facts_stage(out_dir, n, "docs", subjects, seed)


def generate_books(out_dir, n: int = 3, seed: int = 0) -> Path:
    subjects = [("chapter-1", "The hero leaves home"), ("chapter-2", "The hero meets a guide"),
                ("chapter-3", "The hero returns")]
    return _facts_stage(out_dir, n, "book", subjects, seed)


def generate_wikipedia(out_dir, n: int = 3, seed: int = 0) -> Path:
    subjects = [("Paris", "Capital of France"), ("Nile", "A river in Africa"), ("Everest", "The highest mountain")]
    return _facts_stage(out_dir, n, "wiki", subjects, seed)


def generate_hierarchy(out_dir, n: int = 1, seed: int = 0) -> Path:
    """Root documents whose reference tables name section children (depth 2)."""
    documents, references, questions = [], [], []
    for index in range(1, max(n, 1) + 1):
        root = f"memory://project/p{index}"
        section = f"{root}#Authentication"
        detail = f"{section}.details"
        minutes = 30 + index
        documents += [
            {"id": f"p{index}", "uri": root, "title": f"p{index}", "text": f"Project p{index}. Auth is in <REF_1>.",
             "reference_table": {"<REF_1>": section}},
            {"id": f"p{index}a", "uri": section, "title": "Authentication", "text": "Details are in <REF_1>.",
             "reference_table": {"<REF_1>": detail}},
            {"id": f"p{index}d", "uri": detail, "title": "details", "text": f"JWT expiration is {minutes} minutes."},
        ]
        references.append({"id": index, "token": f"<REF_{index}>", "uri": root})
        questions.append({"id": f"h{index}", "prompt": f"What is the JWT expiration? <REF_{index}>",
                          "answer": f"{minutes} minutes", "expected_ref_ids": [index],
                          "expected_anchors": ["Authentication"]})
    return _write_stage(out_dir, documents, references, questions)
