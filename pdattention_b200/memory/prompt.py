"""Long prompts: a bounded direct tail plus an implicit ``#__head`` reference.

Same split contract as ``src/pra_torch/prompt.py:13-231``: the last
``effective_prompt_direct_tokens`` stay direct; overflow follows ``truncate`` /
``implicit_reference`` / ``error``; the head is encoded as a row-local
reference with its own chunk cap (``max_prompt_gists``) and historical
positions continue when the whole history fits natively.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from .cache import PRAMemoryCache, PRASimpleMemoryCache

IMPLICIT_PROMPT_HEAD_URI = "pra://implicit/prompt/head"
IMPLICIT_PROMPT_HEAD_NAME = "#__head"


@dataclass(frozen=True)
class PreparedPrompt:
    direct_ids: tuple[int, ...]
    implicit_ids: tuple[int, ...]
    total_tokens: int
    direct_limit: int
    overflow_mode: str

    @property
    def overflowed(self) -> bool:
        return bool(self.implicit_ids) or self.total_tokens > self.direct_limit


@dataclass(frozen=True)
class PromptPreparationStats:
    total_tokens: int
    direct_tokens: int
    implicit_tokens: int
    implicit_chunks: int
    implicit_gists: int

    def as_metrics(self) -> dict[str, float]:
        return {"prompt_total_tokens": float(self.total_tokens), "prompt_direct_tokens": float(self.direct_tokens),
                "prompt_implicit_tokens": float(self.implicit_tokens),
                "prompt_implicit_chunks": float(self.implicit_chunks),
                "prompt_implicit_gists": float(self.implicit_gists)}


@dataclass
class PreparedPromptBatch:
    input_ids: torch.Tensor
    attention_mask: torch.Tensor
    labels: torch.Tensor | None
    position_offsets: torch.Tensor
    caches: list[PRAMemoryCache]
    splits: list[PreparedPrompt]
    stats: list[PromptPreparationStats]


def prepare_prompt_for_pra(input_ids: Sequence[int] | torch.Tensor, config) -> PreparedPrompt:
    ids = tuple(int(t) for t in input_ids)
    limit = int(config.effective_prompt_direct_tokens)
    mode = config.prompt_overflow_mode
    if len(ids) <= limit:
        return PreparedPrompt(ids, (), len(ids), limit, mode)
    if mode == "error":
        raise ValueError(f"Prompt has {len(ids)} tokens, exceeding direct limit {limit}.")
    if mode == "truncate":
        return PreparedPrompt(ids[-limit:], (), len(ids), limit, "truncate")
    if mode != "implicit_reference":
        raise ValueError(f"Unsupported prompt_overflow_mode: {mode}")
    return PreparedPrompt(ids[-limit:], ids[:-limit], len(ids), limit, "implicit_reference")


def _valid_ids(values: torch.Tensor, mask: torch.Tensor | None) -> list[int]:
    if mask is None:
        return [int(v) for v in values]
    return [int(v) for v, keep in zip(values, mask) if bool(keep)]


def _source_rows(input_ids, attention_mask, labels, metadata):
    ids_rows, label_rows = [], ([] if labels is not None else None)
    for row in range(input_ids.shape[0]):
        item = metadata[row] if metadata is not None else {}
        mask = attention_mask[row] if attention_mask is not None else None
        ids = item.get("full_input_ids")
        ids_rows.append([int(v) for v in (ids if ids is not None else _valid_ids(input_ids[row], mask))])
        if label_rows is not None:
            lab = item.get("full_labels")
            label_rows.append([int(v) for v in (lab if lab is not None else _valid_ids(labels[row], mask))])
    return ids_rows, label_rows


def _pad_rows(rows, *, value, device, dtype):
    if not rows or any(not r for r in rows):
        raise ValueError("Prompt preparation requires at least one token per batch row.")
    width = max(len(r) for r in rows)
    out = torch.full((len(rows), width), value, dtype=dtype)
    mask = torch.zeros((len(rows), width), dtype=torch.long)
    for i, r in enumerate(rows):
        out[i, : len(r)] = torch.tensor(r, dtype=dtype)
        mask[i, : len(r)] = 1
    return out.to(device), mask.to(device)


def head_metadata(row: int, split: PreparedPrompt, max_prompt_gists) -> dict:
    return {"implicit": True, "source": "prompt", "kind": "head", "display_name": IMPLICIT_PROMPT_HEAD_NAME,
            "prompt_row": row, "prompt_total_tokens": split.total_tokens, "prompt_direct_tokens": len(split.direct_ids),
            "prompt_implicit_tokens": len(split.implicit_ids), "max_prompt_gists": max_prompt_gists}


def prepare_prompt_batch_for_pra(model, tokenizer, input_ids: torch.Tensor, *, attention_mask=None, labels=None,
                                 metadata: list[dict] | None = None, caches: list[PRAMemoryCache] | None = None,
                                 pad_token_id: int = 0) -> PreparedPromptBatch:
    """Split every row, right-pad the direct tails and encode each row's implicit head."""
    if input_ids.ndim != 2:
        raise ValueError(f"Expected input_ids [batch,tokens], got {tuple(input_ids.shape)}.")
    batch = int(input_ids.shape[0])
    if metadata is not None and len(metadata) != batch:
        raise ValueError("Prompt metadata must align with input batch rows.")
    caches = caches if caches is not None else [PRASimpleMemoryCache() for _ in range(batch)]
    if len(caches) != batch:
        raise ValueError("Prompt caches must align with input batch rows.")
    cfg = model.cfg
    src_ids, src_labels = _source_rows(input_ids, attention_mask, labels, metadata)
    splits = [prepare_prompt_for_pra(row, cfg) for row in src_ids]
    direct, mask = _pad_rows([list(s.direct_ids) for s in splits], value=pad_token_id, device=input_ids.device,
                             dtype=input_ids.dtype)
    padded_labels = None
    if src_labels is not None:
        tails = [row[-len(s.direct_ids):] for row, s in zip(src_labels, splits)]
        padded_labels, _ = _pad_rows(tails, value=pad_token_id, device=labels.device, dtype=labels.dtype)
    heads = [(row, split) for row, split in enumerate(splits) if split.implicit_ids]
    for cache in caches:
        if hasattr(cache, "invalidate"):
            cache.invalidate(IMPLICIT_PROMPT_HEAD_URI)
    encode_many = getattr(model, "encode_prompt_heads", None)
    entries = {}
    if heads:
        if encode_many is not None:
            entries = encode_many([(row, split) for row, split in heads], tokenizer, input_ids.device)
        else:
            for row, split in heads:
                entries[row] = model.encode_reference_tokens_to_cache(
                    IMPLICIT_PROMPT_HEAD_URI, split.implicit_ids, tokenizer, input_ids.device,
                    metadata=head_metadata(row, split, cfg.max_prompt_gists), max_chunks=cfg.max_prompt_gists,
                    use_configured_max_chunks=False, max_chunk_tokens=cfg.effective_model_max_context_tokens,
                    historical_encoding=(cfg.prompt_position_mode == "historical"))
    stats = []
    for row, (split, cache) in enumerate(zip(splits, caches)):
        chunks = gists = 0
        entry = entries.get(row)
        if entry is not None:
            cache.put(entry)
            chunks = int(entry.metadata.get("chunk_count", 0))
            if entry.layer_memory:
                first = entry.layer_memory[min(entry.layer_memory)]
                gists = sum(int(c.routing_gist.k.shape[0]) for c in first.chunks)
        stats.append(PromptPreparationStats(split.total_tokens, len(split.direct_ids), len(split.implicit_ids),
                                            chunks, gists))
    offsets = torch.tensor([cfg.prompt_tail_position_offset(len(s.implicit_ids), len(s.direct_ids)) for s in splits],
                           dtype=torch.long, device=input_ids.device)
    return PreparedPromptBatch(direct, mask, padded_labels, offsets, caches, splits, stats)


__all__ = ["IMPLICIT_PROMPT_HEAD_NAME", "IMPLICIT_PROMPT_HEAD_URI", "PreparedPrompt", "PreparedPromptBatch",
           "PromptPreparationStats", "head_metadata", "prepare_prompt_batch_for_pra", "prepare_prompt_for_pra"]
