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
        out.append(engine.decode_step(out[-1], sample=True))
    return torch.stack(out, dim=1), plan, first


def run_long_prompt_benchmark(*, model: str = "mistral-7b", batch: int = 16, prompt_tokens: int = 131072,
                              direct_window: int = 4096, new_tokens: int = 256, tp=None, seed: int = 0,
                              clocks=None) -> dict:
    """Long-prompt workload: ``batch`` prompts of ``prompt_tokens`` uniform-random ids; the latest
    ``direct_window`` tokens stay direct, the rest become each row's implicit head chunks
    (64 tokens, one mean gist each).  Times the head build, the tail prefill and
    ``new_tokens`` greedy decode steps (CUDA-graph replays after one eager step); device
    time with CUDA events, max over ranks."""
    import statistics
    import time

    from ..models.llama import PRESETS
    from .llama_engine import LlamaWeights, PRALlamaEngine

    rank = tp.rank if tp is not None else 0
    world = tp.world if tp is not None else 1
    device = torch.device("cuda", torch.cuda.current_device())
    cfg = PRESETS[model](chunk_tokens=64, top_k_chunks=16, direct_window=direct_window)
    engine = PRALlamaEngine(LlamaWeights.random(cfg, device, seed=seed, tp_rank=rank, tp_size=world), device, tp=tp)
    gen = torch.Generator().manual_seed(seed + 1)
    prompts = torch.randint(0, cfg.vocab_size, (batch, prompt_tokens), generator=gen).tolist()
    plan = plan_long_prompts(prompts, direct_window, cfg.chunk_tokens, cfg.max_position_embeddings)

    def timed(fn):
        if tp is not None:
            tp.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        out = fn()
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end)
        return out, (tp.max_scalar(ms) if tp is not None else ms)

    _, build_ms = timed(lambda: engine.build_memory(plan.chunks, plan.chunk_lengths, batch_chunks=256))
    engine.set_namespace(plan.ns_start, plan.ns_end)
    first, prefill_ms = timed(lambda: engine.prefill(plan.tails, plan.tail_lengths, new_tokens + 1, row_batch=4,
                                                     position_offset=plan.position_offset))
    tok = first.float().argmax(-1)
    tok = engine.decode_step(tok, sample=True)  # one eager step, then the captured graph
    engine.capture_decode(sample=True)
    steps = []
    if clocks is not None:
        clocks.__enter__()
    for _ in range(new_tokens - 1):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        tok = engine.decode_step_graphed(tok)
        e.record()
        steps.append((s, e))
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.__exit__(None, None, None)
    per_step = [a.elapsed_time(b) for a, b in steps]
    if tp is not None:
        per_step = [tp.max_scalar(x) for x in per_step]
    engine.release_graph()
    decode_s = sum(per_step) / 1000
    head_tokens = int(plan.chunk_lengths.sum())
    return {"prefill_tokens_per_s": batch * prompt_tokens / ((build_ms + prefill_ms) / 1000),
            "head_build_tokens_per_s": head_tokens / (build_ms / 1000),
            "tail_prefill_tokens_per_s": int(plan.tail_lengths.sum()) / (prefill_ms / 1000),
            "decode_tokens_per_s": batch * len(per_step) / decode_s,
            "tpot_p50_ms": statistics.median(per_step), "head_tokens": head_tokens,
            "memory_gb_per_gpu": engine.memory.nbytes() / 1e9, "batch": batch, "prompt_tokens": prompt_tokens,
            "direct_window": direct_window, "new_tokens": new_tokens, "tp": world, "model": model,
            "params_b": cfg.parameter_count() / 1e9, "decode_steps": len(per_step),
            "position_offset": int(plan.position_offset[0])}
