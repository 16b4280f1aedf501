"""Autoregressive generation with streaming implicit-head rollover.

Semantics of ``src/pra_torch/model.py:1091-1305``: every step re-runs the
model over the (bounded) direct window, so every PRA layer re-routes with the
newest token; when the direct window overflows under ``implicit_reference``,
``rollover_unit`` tokens (the routing chunk size, or half the window) migrate
into the row's ``#__head`` reference, which is re-encoded and republished.

This is the object-path definition (CPU, oracle, small models).  The serving
engine for the large models (``pdattention_b200.serving``) keeps a local KV
cache and appends only completed head chunks instead of recomputing.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ..memory.cache import PRABatchedMemoryCache, PRASimpleMemoryCache
from ..memory.prompt import (
    IMPLICIT_PROMPT_HEAD_NAME,
    IMPLICIT_PROMPT_HEAD_URI,
    prepare_prompt_batch_for_pra,
    prepare_prompt_for_pra,
)


def _row_caches(model, batch: int):
    if isinstance(model.pra_cache, PRABatchedMemoryCache):
        return model.pra_cache.row_caches
    if batch == 1:
        return [model.pra_cache]
    if model.pra_cache.is_empty():
        return [PRASimpleMemoryCache() for _ in range(batch)]
    raise ValueError("Batched generation with explicit references requires row-local caches.")


def generate_with_rollover(model, input_ids, max_new_tokens=64, temperature=1.0, use_pra_memory=True, *,
                           tokenizer=None, do_sample=True):
    cfg = model.cfg
    model.eval()
    batch = input_ids.shape[0]
    implicit = cfg.prompt_overflow_mode == "implicit_reference" and use_pra_memory
    if implicit and input_ids.shape[1] + max_new_tokens > cfg.effective_prompt_direct_tokens and tokenizer is None:
        raise ValueError("tokenizer is required for streaming prompt-history rollover.")
    if batch > 1 and not isinstance(model.pra_cache, PRABatchedMemoryCache):
        if not model.pra_cache.is_empty():
            raise ValueError("Batched generation with explicit references requires row-local caches.")
        model.set_pra_cache(PRABatchedMemoryCache([PRASimpleMemoryCache() for _ in range(batch)]))
    caches = model.pra_cache.row_caches if isinstance(model.pra_cache, PRABatchedMemoryCache) else [model.pra_cache]
    for cache in caches:
        if hasattr(cache, "invalidate"):
            cache.invalidate(IMPLICIT_PROMPT_HEAD_URI)

    output_ids = direct_ids = input_ids
    heads = [[] for _ in range(batch)]
    if input_ids.shape[1] > cfg.effective_prompt_direct_tokens:
        if implicit:
            if tokenizer is None:
                raise ValueError("tokenizer is required to build implicit memory for a long prompt.")
            caches = _row_caches(model, batch)
            prepared = prepare_prompt_batch_for_pra(model, tokenizer, input_ids, caches=caches)
            direct_ids = prepared.input_ids
            heads = [list(s.implicit_ids) for s in prepared.splits]
            model.set_pra_cache(caches[0] if len(caches) == 1 else PRABatchedMemoryCache(caches))
        else:
            direct_ids = input_ids.new_tensor([list(prepare_prompt_for_pra(r, cfg).direct_ids) for r in input_ids])

    limit = cfg.effective_prompt_direct_tokens
    unit = max(1, min(int(cfg.routing_chunking_config.chunk_tokens or max(limit // 2, 1)), limit))
    stats = {"rollover_events": 0, "tokens_migrated": 0, "max_direct_tokens_observed": int(direct_ids.shape[1]),
             "max_native_operation_tokens": int(direct_ids.shape[1]), "routing_steps": 0,
             "routing_duration_seconds_total": 0.0, "materialized_memory_tokens_total": 0.0,
             "max_materialized_memory_tokens_observed": 0.0}
    for _ in range(max_new_tokens):
        window = direct_ids[:, -limit:]
        offsets = torch.tensor([cfg.prompt_tail_position_offset(len(h), window.shape[1]) for h in heads],
                               dtype=torch.long, device=window.device)
        logits = model(window, use_pra_memory=use_pra_memory, position_offset=offsets)
        diag = list(model.pra_diagnostics_by_layer().values())
        per_layer = [float(d.get("memory_tokens_materialized", 0.0)) for d in diag]
        if any(d.get("routing_candidates", 0.0) for d in diag):
            stats["routing_steps"] += 1
        stats["routing_duration_seconds_total"] += sum(float(d.get("routing_duration_seconds", 0.0)) for d in diag)
        stats["materialized_memory_tokens_total"] += sum(per_layer) / max(len(per_layer), 1)
        stats["max_materialized_memory_tokens_observed"] = max(stats["max_materialized_memory_tokens_observed"],
                                                               max(per_layer, default=0.0))
        last = logits[:, -1, :] / max(temperature, 1e-6)
        nxt = torch.multinomial(F.softmax(last, dim=-1), 1) if do_sample else last.argmax(dim=-1, keepdim=True)
        direct_ids = torch.cat([direct_ids, nxt], dim=1)
        output_ids = torch.cat([output_ids, nxt], dim=1)
        if direct_ids.shape[1] > limit:
            if cfg.prompt_overflow_mode == "error":
                raise ValueError("Generated direct history exceeded its configured limit.")
            if implicit:
                move = min(unit, int(direct_ids.shape[1]) - 1)
                moved, direct_ids = direct_ids[:, :move], direct_ids[:, move:]
                for row, cache in enumerate(caches):
                    heads[row].extend(int(v) for v in moved[row])
                    if hasattr(cache, "invalidate"):
                        cache.invalidate(IMPLICIT_PROMPT_HEAD_URI)
                    cache.put(model.encode_reference_tokens_to_cache(
                        IMPLICIT_PROMPT_HEAD_URI, heads[row], tokenizer, input_ids.device,
                        metadata={"implicit": True, "source": "prompt", "kind": "streaming_head",
                                  "display_name": IMPLICIT_PROMPT_HEAD_NAME, "prompt_row": row, "streaming": True,
                                  "rollover_events": stats["rollover_events"] + 1,
                                  "tokens_migrated": len(heads[row])},
                        max_chunks=cfg.max_prompt_gists, use_configured_max_chunks=False,
                        max_chunk_tokens=cfg.effective_model_max_context_tokens,
                        historical_encoding=cfg.prompt_position_mode == "historical"))
                stats["rollover_events"] += 1
                stats["tokens_migrated"] += move * int(batch)
            else:
                direct_ids = direct_ids[:, -limit:]
        stats["max_direct_tokens_observed"] = max(stats["max_direct_tokens_observed"], int(direct_ids.shape[1]))
        encoded_max = max((int(c.get(IMPLICIT_PROMPT_HEAD_URI).metadata.get("max_encoding_input_tokens", 0))
                           for c in caches if c.get(IMPLICIT_PROMPT_HEAD_URI) is not None), default=0)
        stats["max_native_operation_tokens"] = max(stats["max_native_operation_tokens"], int(window.shape[1]),
                                                   encoded_max)
    model.last_generation_stats = {
        "generated_tokens": int(max_new_tokens), "direct_tokens": int(direct_ids.shape[1]),
        "head_tokens": sum(len(h) for h in heads), **stats,
        "model_max_context_tokens": cfg.effective_model_max_context_tokens,
    }
    return output_ids
