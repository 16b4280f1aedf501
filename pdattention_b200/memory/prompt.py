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
    """Split one prompt into its direct tail and (``implicit_reference`` mode) its implicit head."""
    ids = tuple(map(int, input_ids))
    limit = int(config.effective_prompt_direct_tokens)
    mode = config.prompt_overflow_mode
    overflow = len(ids) - limit
    if overflow <= 0:
        return PreparedPrompt(ids, (), len(ids), limit, mode)
    if mode not in ("error", "truncate", "implicit_reference"):
        raise ValueError(f"Unsupported prompt_overflow_mode: {mode}")
    if mode == "error":
        raise ValueError(f"Prompt has {len(ids)} tokens, exceeding direct limit {limit}.")
    head = ids[:overflow] if mode == "implicit_reference" else ()
    return PreparedPrompt(ids[overflow:], head, len(ids), limit, mode)


def _row_tokens(values: torch.Tensor, mask: torch.Tensor | None, full) -> list[int]:
    """A row's untruncated tokens from metadata when the collator kept them, else its valid ids."""
    if full is not None:
        return list(map(int, full))
    keep = values if mask is None else values[mask.bool()]
    return keep.tolist()


def _right_pad(rows: list[list[int]], value: int, device, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    if not rows or min(map(len, rows)) == 0:
        raise ValueError("Prompt preparation requires at least one token per batch row.")
    tensors = [torch.tensor(r, dtype=dtype) for r in rows]
    padded = torch.nn.utils.rnn.pad_sequence(tensors, batch_first=True, padding_value=value)
    lengths = torch.tensor([len(r) for r in rows])
    mask = (torch.arange(padded.shape[1])[None, :] < lengths[:, None]).long()
    return padded.to(device), mask.to(device)


def head_metadata(row: int, split: PreparedPrompt, max_prompt_gists) -> dict:
    """Metadata recorded on a row's implicit head entry."""
    return {"implicit": True, "source": "prompt", "kind": "head", "display_name": IMPLICIT_PROMPT_HEAD_NAME,
            "prompt_row": row, "prompt_total_tokens": split.total_tokens, "prompt_direct_tokens": len(split.direct_ids),
            "prompt_implicit_tokens": len(split.implicit_ids), "max_prompt_gists": max_prompt_gists}


def _encode_heads(model, tokenizer, heads: list[tuple[int, PreparedPrompt]], device) -> dict:
    """row -> encoded implicit-head entry (batched when the model can, else one row at a time)."""
    if not heads:
        return {}
    batched = getattr(model, "encode_prompt_heads", None)
    if batched is not None:
        return batched(heads, tokenizer, device)
    cfg = model.cfg
    return {row: model.encode_reference_tokens_to_cache(
                IMPLICIT_PROMPT_HEAD_URI, split.implicit_ids, tokenizer, device,
                metadata=head_metadata(row, split, cfg.max_prompt_gists), max_chunks=cfg.max_prompt_gists,
                use_configured_max_chunks=False, max_chunk_tokens=cfg.effective_model_max_context_tokens,
                historical_encoding=cfg.prompt_position_mode == "historical")
            for row, split in heads}


def _head_sizes(entry) -> tuple[int, int]:
    """(chunks, gists of the first encoded layer) of a head entry."""
    if entry is None:
        return 0, 0
    gists = 0
    if entry.layer_memory:
        gists = sum(int(c.routing_gist.k.shape[0]) for c in entry.layer_memory[min(entry.layer_memory)].chunks)
    return int(entry.metadata.get("chunk_count", 0)), gists


def prepare_prompt_batch_for_pra(model, tokenizer, input_ids: torch.Tensor, *, attention_mask=None, labels=None,
                                 metadata: list[dict] | None = None, caches: list[PRAMemoryCache] | None = None,
                                 pad_token_id: int = 0) -> PreparedPromptBatch:
    """Split every row, right-pad the direct tails (and their labels), and put each row's encoded
    implicit head into that row's cache (replacing an earlier head)."""
    if input_ids.ndim != 2:
        raise ValueError(f"Expected input_ids [batch,tokens], got {tuple(input_ids.shape)}.")
    batch = int(input_ids.shape[0])
    if metadata is not None and len(metadata) != batch:
        raise ValueError("Prompt metadata must align with input batch rows.")
    caches = [PRASimpleMemoryCache() for _ in range(batch)] if caches is None else caches
    if len(caches) != batch:
        raise ValueError("Prompt caches must align with input batch rows.")
    cfg = model.cfg
    items = metadata if metadata is not None else [{}] * batch
    masks = attention_mask if attention_mask is not None else [None] * batch
    token_rows = [_row_tokens(input_ids[r], masks[r], items[r].get("full_input_ids")) for r in range(batch)]
    splits = [prepare_prompt_for_pra(row, cfg) for row in token_rows]
    direct, mask = _right_pad([list(s.direct_ids) for s in splits], pad_token_id, input_ids.device, input_ids.dtype)
    padded_labels = None
    if labels is not None:
        label_rows = [_row_tokens(labels[r], masks[r], items[r].get("full_labels")) for r in range(batch)]
        padded_labels, _ = _right_pad([row[-len(s.direct_ids):] for row, s in zip(label_rows, splits)],
                                      pad_token_id, labels.device, labels.dtype)
    for cache in caches:
        if hasattr(cache, "invalidate"):
            cache.invalidate(IMPLICIT_PROMPT_HEAD_URI)
    entries = _encode_heads(model, tokenizer, [(r, s) for r, s in enumerate(splits) if s.implicit_ids],
                            input_ids.device)
    stats = []
    for row, split in enumerate(splits):
        entry = entries.get(row)
        if entry is not None:
            caches[row].put(entry)
        stats.append(PromptPreparationStats(split.total_tokens, len(split.direct_ids), len(split.implicit_ids),
                                            *_head_sizes(entry)))
    offsets = torch.tensor([cfg.prompt_tail_position_offset(len(s.implicit_ids), len(s.direct_ids)) for s in splits],
                           dtype=torch.long, device=input_ids.device)
    return PreparedPromptBatch(direct, mask, padded_labels, offsets, caches, splits, stats)


__all__ = ["IMPLICIT_PROMPT_HEAD_NAME", "IMPLICIT_PROMPT_HEAD_URI", "PreparedPrompt", "PreparedPromptBatch",
           "PromptPreparationStats", "head_metadata", "prepare_prompt_batch_for_pra", "prepare_prompt_for_pra"]
