"""WikiText-derived reference stages (continuation and fixed-target history partitions).

Each qualifying WikiText train row (a paragraph of at least ``min_words``
words) becomes one example: its words are cut into equal parts, the earlier
parts become references and the held-out tail supplies the prompt and the
answer.  Three layouts, matching the reference's stages field for field
(``src/data/datasets.py:328-659``):

* ``wikitext2_references`` (v1): ``<REF_1> .. <REF_n>`` in order, answer = the
  last 8-16 tail words;
* ``wikitext2_references_v2``: reference ids shuffled, candidate order
  shuffled, a lead-in of up to 16 tail words in the prompt and only the last
  history part labelled relevant;
* ``wikitext2_nativekv_fixed_target``: prompt and target fixed (the last
  ``local_tail_words`` + ``target_words`` words), only the history before them
  is partitioned into ``split_count - 1`` implicit-history references.

This framework never downloads: the rows come from a local copy of the corpus
(``corpus_path``: the raw ``wiki.train.raw`` file, or a directory holding it)
or from the ``datasets`` package's cache when that package is importable.
Rows are the corpus lines; a row counts when its stripped text is non-empty,
exactly as the Hugging Face split exposes them.
"""

from __future__ import annotations

import hashlib
import random
from collections.abc import Iterable
from pathlib import Path

from ..datasets import write_jsonl

WIKITEXT_NAMES = ("wikitext-2-raw-v1", "wikitext-103-raw-v1")
_RAW_FILES = ("wiki.train.raw", "train.txt", "wiki.train.tokens")


def wikitext_train_rows(dataset_name: str = "wikitext-2-raw-v1", *, corpus_path=None, cache_dir=None) -> list[str]:
    """The train split's rows (one string per corpus line)."""
    if dataset_name not in WIKITEXT_NAMES:
        raise ValueError(f"Unsupported WikiText dataset: {dataset_name}")
    if corpus_path is not None:
        path = Path(corpus_path)
        if path.is_dir():
            found = [path / name for name in _RAW_FILES if (path / name).exists()]
            if not found:
                raise FileNotFoundError(f"no {' / '.join(_RAW_FILES)} under {path}")
            path = found[0]
        return path.read_text(encoding="utf-8").splitlines()
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise RuntimeError("WikiText stages need corpus_path= (a local wiki.train.raw) or the 'datasets' "
                           "package with a cached copy of Salesforce/wikitext") from exc
    split = load_dataset("Salesforce/wikitext", dataset_name, cache_dir=str(cache_dir) if cache_dir else None)
    return [str(r["text"]) for r in split["train"]]


def wikitext_documents(rows: Iterable, *, max_documents: int | None = None) -> list[str]:
    """Non-empty rows, stripped (rows may be strings or ``{"text": ...}`` records)."""
    docs = []
    for row in rows:
        text = str(row["text"] if isinstance(row, dict) else row).strip()
        if text:
            docs.append(text)
    return docs if max_documents is None else docs[:max_documents]


def _qualifying(rows, min_words: int, seed: int) -> tuple[random.Random, list[tuple[int, list[str]]]]:
    """(source index, words) of every document with ``>= min_words`` words, shuffled by a
    generator seeded ``seed`` (returned, since v2 keeps drawing from it)."""
    docs = [(i, text.split()) for i, text in enumerate(wikitext_documents(rows))]
    picked = [(i, w) for i, w in docs if len(w) >= min_words]
    rng = random.Random(seed)
    rng.shuffle(picked)
    return rng, picked


def _equal_parts(words: list[str], part_count: int) -> tuple[int, list[str], list[str]]:
    """``part_count - 1`` leading parts of ``len // part_count`` words and the tail after them."""
    size = max(1, len(words) // part_count)
    refs = part_count - 1
    return size, [" ".join(words[j * size:(j + 1) * size]) for j in range(refs)], words[refs * size:]


def _check_counts(split_count, max_reference_parts) -> None:
    if split_count is not None and split_count < 2:
        raise ValueError("split_count must include at least one reference and one tail")
    if max_reference_parts < 1:
        raise ValueError("max_reference_parts must be at least 1")


def _save(stage_dir: Path, documents, references, questions) -> Path:
    for name, rows in (("documents", documents), ("references", references), ("questions", questions)):
        write_jsonl(stage_dir / f"{name}.jsonl", rows)
    return stage_dir


def generate_wikitext_reference_dataset(data_dir, *, dataset_name: str = "wikitext-2-raw-v1", max_examples: int = 128,
                                        max_reference_parts: int = 5, split_count: int | None = None, seed: int = 7,
                                        min_words: int = 80, cache_dir=None, corpus_path=None) -> Path:
    """``wikitext2_references``: the tail continues the referenced parts (v1 layout)."""
    _check_counts(split_count, max_reference_parts)
    data_dir = Path(data_dir)
    rows = wikitext_train_rows(dataset_name, corpus_path=corpus_path, cache_dir=cache_dir or data_dir / ".hf_cache")
    _, picked = _qualifying(rows, min_words, seed)
    documents, references, questions = [], [], []
    for ex, (_, words) in enumerate(picked[:max_examples]):
        n_parts = split_count or (2 + ex % max_reference_parts)
        size, parts, tail = _equal_parts(words, n_parts)
        n_refs = n_parts - 1
        answer_size = max(8, min(16, len(tail) // 3))
        uris = []
        for rid, text in enumerate(parts, start=1):
            uri = f"wikitext://{dataset_name}/{ex}/part-{rid}"
            uris.append(uri)
            documents.append({"id": f"wiki-{ex}-{rid}", "uri": uri, "title": f"WikiText {ex} part {rid}",
                              "text": text})
            references.append({"id": rid, "token": f"<REF_{rid}>", "uri": uri, "metadata": {"dataset": dataset_name}})
        ids = list(range(1, n_refs + 1))
        questions.append({
            "id": f"wikitext-ref-{ex}",
            "prompt": " ".join(f"<REF_{i}>" for i in ids) + " Continue the referenced WikiText passage:",
            "answer": " ".join(tail[-answer_size:]), "reference_uris": uris, "expected_ref_ids": ids,
            "expected_anchors": [], "source_wikitext_entry": ex,
            "part_boundaries": [j * size for j in range(n_parts + 1)],
            "part_identifiers": [f"part-{i}" for i in ids], "candidate_reference_parts": ids,
            "intended_relevant_parts": ids, "tail_span": [len(words) - answer_size, len(words)],
            "token_distance": max(len(words) - n_refs * size, 0), "number_of_parts": n_parts,
            "split_count": n_parts, "reference_count": n_refs, "local_context_sufficient": False,
            "reference_relation": "indirect_natural_continuation"})
    return _save(data_dir / "wikitext2_references", documents, references, questions)


def generate_wikitext_reference_dataset_v2(data_dir, *, dataset_name: str = "wikitext-2-raw-v1",
                                           max_examples: int = 512, max_reference_parts: int = 5,
                                           split_count: int | None = None, seed: int = 1729, min_words: int = 80,
                                           cache_dir=None, corpus_path=None) -> Path:
    """``wikitext2_references_v2``: shuffled reference ids and candidate order, a lead-in in the
    prompt, only the part right before the tail labelled relevant."""
    _check_counts(split_count, max_reference_parts)
    data_dir = Path(data_dir)
    rows = wikitext_train_rows(dataset_name, corpus_path=corpus_path, cache_dir=cache_dir or data_dir / ".hf_cache")
    rng, picked = _qualifying(rows, min_words, seed)
    documents, references, questions = [], [], []
    for ex, (src, words) in enumerate(picked[:max_examples]):
        n_parts = split_count or (2 + ex % max_reference_parts)
        _, parts, tail = _equal_parts(words, n_parts)
        n_refs = n_parts - 1
        answer_size = min(12, max(4, len(tail) // 3))
        lead = min(16, max(1, len(tail) - answer_size))
        ids = list(range(1, n_refs + 1))
        rng.shuffle(ids)
        slots = list(enumerate(zip(parts, ids), start=1))  # (chronological part, (text, reference id))
        relevant = slots[-1][1][1]
        rng.shuffle(slots)
        uris, order = [], []
        for chrono, (text, rid) in slots:
            uri = f"wikitext://{dataset_name}/{src}/part-{chrono}"
            uris.append(uri)
            order.append(rid)
            documents.append({"id": f"wiki-{src}-{chrono}", "uri": uri,
                              "title": f"WikiText source {src} part {chrono}", "text": text})
            references.append({"id": rid, "token": f"<REF_{rid}>", "uri": uri,
                               "metadata": {"dataset": dataset_name, "source_entry_id": src,
                                            "chronological_part": chrono, "generation_version": "wikitext_refs_v2"}})
        questions.append({
            "id": f"wikitext-ref-v2-{src}",
            "prompt": " ".join(f"<REF_{r}>" for r in order)
            + " Continue the referenced WikiText passage after this lead-in: " + " ".join(tail[:lead]),
            "answer": " ".join(tail[lead: lead + answer_size]), "reference_uris": uris,
            "expected_ref_ids": [relevant], "expected_anchors": [], "source_entry_id": src, "part_ids": order,
            "relevant_part_ids": [relevant], "target_part_id": f"tail-{src}", "num_parts": n_parts,
            "split_count": n_parts, "reference_count": n_refs, "reference_distance_tokens": lead,
            "local_context_sufficient": False, "dependency_type": "indirect_continuation",
            "generation_version": "wikitext_refs_v2", "candidate_order_randomized": True})
    return _save(data_dir / "wikitext2_references_v2", documents, references, questions)


def generate_wikitext_nativekv_fixed_target_dataset(data_dir, *, split_count: int,
                                                    dataset_name: str = "wikitext-2-raw-v1", max_examples: int = 128,
                                                    seed: int = 1729, min_words: int = 160, local_tail_words: int = 16,
                                                    target_words: int = 12, cache_dir=None, corpus_path=None) -> Path:
    """``wikitext2_nativekv_fixed_target``: fixed local tail and target; the history before
    them is cut into ``split_count - 1`` implicit-history references."""
    if split_count not in (2, 3, 5, 8, 16, 32, 64):
        raise ValueError("split_count must be one of 2, 3, 5, 8, 16, 32, or 64")
    if local_tail_words <= 0 or target_words <= 0:
        raise ValueError("local_tail_words and target_words must be positive")
    data_dir = Path(data_dir)
    rows = wikitext_train_rows(dataset_name, corpus_path=corpus_path, cache_dir=cache_dir or data_dir / ".hf_cache")
    _, picked = _qualifying(rows, min_words, seed)
    n_refs = split_count - 1
    documents, references, questions = [], [], []
    for src, words in picked[:max_examples]:
        cut = len(words) - target_words - local_tail_words
        history, local, target = words[:cut], words[cut: cut + local_tail_words], words[-target_words:]
        if len(history) < n_refs:
            continue
        bounds = [j * len(history) // n_refs for j in range(n_refs + 1)]
        uris = []
        for j in range(n_refs):
            lo, hi = bounds[j], bounds[j + 1]
            uri = f"wikitext://{dataset_name}/{src}/native-history-{j + 1}-of-{n_refs}"
            uris.append(uri)
            documents.append({"id": f"native-{src}-{j + 1}", "uri": uri,
                              "title": f"WikiText source {src} history {j + 1}", "text": " ".join(history[lo:hi])})
            references.append({"id": j + 1, "token": f"<REF_{j + 1}>", "uri": uri,
                               "metadata": {"dataset": dataset_name, "source_entry_id": src,
                                            "implicit_reference": "#__head", "history_word_span": [lo, hi]}})
        prompt, answer = " ".join(local), " ".join(target)
        questions.append({
            "id": f"wikitext-native-{src}", "prompt": prompt, "answer": answer, "reference_uris": uris,
            "expected_ref_ids": list(range(1, n_refs + 1)), "source_entry_id": src, "split_count": split_count,
            "reference_count": n_refs, "history_word_count": len(history), "history_boundaries": bounds,
            "local_tail_word_count": len(local), "target_word_count": len(target),
            "fixed_target_id": hashlib.sha256(f"{src}\n{prompt}\n{answer}".encode("utf-8")).hexdigest(),
            "implicit_reference_uri": "#__head", "generation_version": "wikitext_nativekv_fixed_target_v1"})
    return _save(data_dir / "wikitext2_nativekv_fixed_target", documents, references, questions)
