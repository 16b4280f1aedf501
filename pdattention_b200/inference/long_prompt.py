"""Long prompts through an implicit head reference (PRA Llama-family engine).

A prompt longer than the direct window keeps its latest ``direct_window`` tokens in
direct causal attention; the earlier tokens become the chunks of the row's implicit
reference ``pra://implicit/prompt/head`` (``chunk_tokens`` each, the last one
shorter), which only that row's routing can read.  This is the reference's prompt
overflow path (``src/pra_torch/prompt.py:125-231``, positions as in
``config.py:194-202``): in ``historical`` mode the direct tail continues the head's
positions while head + tail still fit the model's native positions, otherwise (and in
``restart`` mode) the tail starts at position 0.

The head chunks of every row are built in one batched memory encode, then the tails
are prefilled and decoded by the engine as usual.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

IMPLICIT_HEAD_URI = "pra://implicit/prompt/head"


@dataclass
class LongPromptPlan:
    chunks: torch.Tensor          # [C, chunk_tokens] head chunks of every row (padded)
    chunk_lengths: torch.Tensor   # [C]
    ns_start: torch.Tensor        # [B] row b reads chunks [ns_start[b], ns_end[b])
    ns_end: torch.Tensor
    tails: torch.Tensor           # [B, W] direct tokens (left-aligned, padded)
    tail_lengths: torch.Tensor    # [B]
    position_offset: torch.Tensor  # [B] position of each tail's first token
    chunk_ids: list = field(default_factory=list)  # per chunk: "pra://implicit/prompt/head#chunk=i" per row


def plan_long_prompts(prompts: list[list[int]], direct_window: int, chunk_tokens: int, max_positions: int,
                      position_mode: str = "historical", pad_id: int = 0) -> LongPromptPlan:
    if position_mode not in ("historical", "restart"):
        raise ValueError("position_mode must be 'historical' or 'restart'")
    chunks, lengths, starts, ends, tails, offsets, ids = [], [], [], [], [], [], []
    for row in prompts:
        row = [int(t) for t in row]
        head, tail = row[: max(0, len(row) - direct_window)], row[max(0, len(row) - direct_window):]
        starts.append(len(chunks))
        for i, c0 in enumerate(range(0, len(head), chunk_tokens)):
            piece = head[c0: c0 + chunk_tokens]
            chunks.append(piece + [pad_id] * (chunk_tokens - len(piece)))
            lengths.append(len(piece))
            ids.append(f"{IMPLICIT_HEAD_URI}#chunk={i}")
        ends.append(len(chunks))
        tails.append(tail)
        legal = len(head) + len(tail) <= max_positions
        offsets.append(len(head) if position_mode == "historical" and legal else 0)
    width = max((len(t) for t in tails), default=1)
    tail_t = torch.full((len(prompts), max(width, 1)), pad_id, dtype=torch.long)
    for b, t in enumerate(tails):
        tail_t[b, : len(t)] = torch.tensor(t, dtype=torch.long)
    chunk_t = torch.tensor(chunks, dtype=torch.long) if chunks else torch.zeros((0, chunk_tokens), dtype=torch.long)
    return LongPromptPlan(chunk_t, torch.tensor(lengths, dtype=torch.int32), torch.tensor(starts, dtype=torch.int32),
                          torch.tensor(ends, dtype=torch.int32), tail_t,
                          torch.tensor([len(t) for t in tails], dtype=torch.int32),
                          torch.tensor(offsets, dtype=torch.int32), ids)


@torch.no_grad()
def long_prompt_generate(engine, prompts: list[list[int]], max_new_tokens: int, *, direct_window: int | None = None,
                         position_mode: str = "historical", row_batch: int | None = None,
                         build_chunks: int = 256) -> tuple[torch.Tensor, LongPromptPlan, torch.Tensor]:
    """Greedy generation for prompts longer than the direct window.  Returns (new token
    ids ``[B, max_new_tokens]``, the plan, the logits of each prompt's last token)."""
    cfg = engine.cfg
    window = direct_window or cfg.direct_window
    plan = plan_long_prompts(prompts, window, cfg.chunk_tokens, cfg.max_position_embeddings, position_mode)
    if plan.chunks.shape[0]:
        engine.build_memory(plan.chunks, plan.chunk_lengths, batch_chunks=build_chunks)
        engine.set_namespace(plan.ns_start, plan.ns_end)
    else:
        engine.memory = None
    first = engine.prefill(plan.tails, plan.tail_lengths, max_new_tokens, row_batch=row_batch,
                           position_offset=plan.position_offset)
    out = [first.float().argmax(-1)]
    for _ in range(max_new_tokens - 1):
        out.append(engine.decode_step(out[-1]).float().argmax(-1))
    return torch.stack(out, dim=1), plan, first
