"""Controlled memory interventions (``evaluate_reference_ablation``).

Sixteen conditions of ``src/pra_torch/pra_train.py:648-1103``: ``valid`` routes
normally; ``disabled`` / ``native_disabled`` bypass memory; ``empty`` keeps the
branch with no entries; ``shuffled`` / ``irrelevant`` swap URI sets across
examples; ``oracle`` exposes only target URIs; ``oracle_chunks`` keeps only
target chunks; ``shuffled_chunks`` / ``irrelevant_chunks`` rotate detail K/V
between chunks while keeping their gists; ``full_reference`` /
``selected_chunks`` / ``gist_only`` switch the materialisation mode;
``native_all`` / ``native_oracle`` materialise every chunk (all URIs / target
URIs).  Each example runs a batch-1 forward; per-example records carry loss,
selection, sparsity and latency fields used by the systems benchmarks.
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F

from .memory.cache import PRASimpleMemoryCache
from .memory.services import build_cache_from_metadata
from .runtime.metrics import perplexity
from .runtime.train import move_batch

CONDITIONS = ("valid", "disabled", "shuffled", "irrelevant", "empty", "oracle", "full_reference", "selected_chunks",
              "oracle_chunks", "shuffled_chunks", "irrelevant_chunks", "gist_only", "native_all", "native_oracle",
              "native_disabled", "native_shuffled")


def _expected_uris(item) -> set[str]:
    explicit = set(item.get("target_reference_uris") or [])
    if explicit:
        return explicit
    ids = set(item.get("target_reference_ids") or [])
    return {ref.uri for ref in item["references"] if ref.id in ids}


def _intervened_metadata(condition, item, reference_sets, pool, cursor, offset, cfg):
    if condition in {"shuffled", "native_shuffled"}:
        return {**item, "references": reference_sets[(cursor + offset) % len(reference_sets)]}
    if condition == "irrelevant":
        own = {r.uri for r in item["references"]}
        start = (cursor + offset) % max(len(pool), 1)
        others = [r for r in pool[start:] + pool[:start] if r.uri not in own]
        return {**item, "references": others[: len(item["references"])]}
    if condition in {"oracle", "native_oracle"} and cfg.reference_encoding_strategy == "independent":
        ids = set(item["target_reference_ids"])
        return {**item, "references": [r for r in item["references"] if r.id in ids]}
    return item


def _intervene_chunks(condition, cache, item, n_layers):
    if condition == "oracle_chunks":
        keep = set(item.get("target_chunk_ids") or [])
        if keep:
            for entry in cache.all_entries():
                for memory in entry.layer_memory.values():
                    memory.chunks[:] = [c for c in memory.chunks if c.chunk_id in keep]
    elif condition in {"shuffled_chunks", "irrelevant_chunks"}:
        for layer_id in range(n_layers):
            chunks = [c for e in cache.all_entries() if layer_id in e.layer_memory
                      for c in e.layer_memory[layer_id].chunks]
            if len(chunks) > 1:
                payloads = [c.token_kv for c in chunks]
                for chunk, kv in zip(chunks, payloads[1:] + payloads[:1]):
                    chunk.token_kv = kv


def evaluate_reference_ablation(*, model, loader, tokenizer, device: str, condition: str, resolver_config=None,
                                cache_config=None, collect_per_example: bool = False,
                                encoded_entry_cache: dict | None = None) -> dict:
    if condition not in CONDITIONS:
        raise ValueError(f"Unsupported reference condition: {condition}")
    cfg = model.cfg
    if condition.startswith("native_") and cfg.memory_transport != "native_kv":
        raise ValueError(f"{condition} requires memory_transport='native_kv'")
    was_training = model.training
    model.eval()
    reference_sets = ([item["references"] for batch in loader for item in batch["metadata"]]
                      if condition in {"shuffled", "irrelevant", "native_shuffled"} else [])
    pool = [r for refs in reference_sets for r in refs]
    offset = max(len(reference_sets) // 2, 1)
    saved = (cfg.detail_materialization, cfg.top_k_references, cfg.top_k_chunks_per_reference, cfg.trigger_threshold)
    if condition in {"native_all", "native_oracle"}:
        cfg.top_k_references = cfg.top_k_chunks_per_reference = 1_000_000
        cfg.trigger_threshold = float("-inf")
        cfg.detail_materialization = "full_reference"
    if condition in {"full_reference", "selected_chunks", "gist_only"}:
        cfg.detail_materialization = condition
    materialization = cfg.detail_materialization
    loss_sum = correct = token_count = 0
    per_example, cursor = [], 0
    t_start = time.perf_counter()
    try:
        with torch.no_grad():
            for batch in loader:
                moved = move_batch(batch, device)
                for index, item in enumerate(batch["metadata"]):
                    t_item = time.perf_counter()
                    memory_on = condition not in {"disabled", "native_disabled"}
                    if condition in {"disabled", "empty", "native_disabled"}:
                        model.clear_pra_cache()
                    else:
                        metadata = _intervened_metadata(condition, item, reference_sets, pool, cursor, offset, cfg)
                        uris = [r.uri for r in metadata["references"]]
                        if encoded_entry_cache is not None and all(u in encoded_entry_cache for u in uris):
                            cache = PRASimpleMemoryCache()
                            for u in uris:
                                cache.put(encoded_entry_cache[u])
                            model.set_pra_cache(cache)
                        else:
                            cache = build_cache_from_metadata(model, tokenizer, [metadata], device,
                                                              resolver_config=resolver_config,
                                                              cache_config=cache_config)
                            if encoded_entry_cache is not None:
                                encoded_entry_cache.update(cache.entries)
                        if condition in {"oracle", "native_oracle"} and cfg.reference_encoding_strategy != "independent":
                            filtered = PRASimpleMemoryCache()
                            for u in _expected_uris(item):
                                if cache.get(u) is not None:
                                    filtered.put(cache.get(u))
                            cache = filtered
                            model.set_pra_cache(cache)
                        _intervene_chunks(condition, cache, item, cfg.n_layers)
                    position_offset = 0
                    if cfg.prompt_position_mode == "historical" and memory_on:
                        position_offset = sum(len(tokenizer.encode(str(r.metadata.get("text", ""))))
                                              for r in item.get("references") or [])
                    logits = model(moved["input_ids"][index:index + 1], use_pra_memory=memory_on,
                                   position_offset=position_offset)
                    labels = moved["labels"][index:index + 1]
                    valid = labels.ne(0)
                    count = int(valid.sum().item())
                    item_loss = float(F.cross_entropy(logits.reshape(-1, logits.size(-1)), labels.reshape(-1),
                                                      ignore_index=0, reduction="sum").cpu())
                    item_correct = int((logits.argmax(dim=-1).eq(labels) & valid).sum().item())
                    loss_sum, correct, token_count = loss_sum + item_loss, correct + item_correct, token_count + count
                    if collect_per_example:
                        per_example.append(_example_record(model, item, moved, index, condition, item_loss,
                                                           item_correct, count, tokenizer, t_item))
                    cursor += 1
    finally:
        cfg.detail_materialization, cfg.top_k_references, cfg.top_k_chunks_per_reference, cfg.trigger_threshold = saved
        if was_training:
            model.train()
    loss = loss_sum / max(token_count, 1)
    result = {"condition": condition, "loss": loss, "perplexity": perplexity(loss),
              "token_accuracy": correct / max(token_count, 1), "tokens": token_count,
              "duration_seconds": max(time.perf_counter() - t_start, 1e-9),
              "detail_materialization": materialization, "ablation": condition,
              "memory_transport": cfg.memory_transport}
    if collect_per_example:
        result["per_example"] = per_example
    return result


def _example_record(model, item, moved, index, condition, item_loss, item_correct, count, tokenizer, t_item) -> dict:
    from .pra_train import _complete_reference_rank_metrics

    cfg = model.cfg
    layer_hits = {int(l): (rows[0] if rows else []) for l, rows in model.selected_chunks_by_layer().items()}
    rankings = {int(l): (rows[0] if rows else []) for l, rows in model.routing_rankings_by_layer().items()}
    hits = [h for row in layer_hits.values() for h in row]
    per_layer = [sum(h.selected_token_count for h in row) for row in layer_hits.values()]
    retrieved = sum(per_layer) / len(per_layer) if per_layer else 0.0
    local = int(moved.get("attention_mask", moved["input_ids"].ne(0))[index:index + 1].sum().item())
    displaced = sum(len(tokenizer.encode(str(r.metadata.get("text", "")))) for r in item.get("references") or [])
    diag = list(model.pra_diagnostics_by_layer().values())
    selected = sorted({h.reference_uri for h in hits})
    targets = _expected_uris(item)
    scores = [float(h.chunk_score) for h in hits]
    return {
        "example_id": str(item["id"]), "condition": condition, "loss": item_loss / max(count, 1),
        "perplexity": perplexity(item_loss / max(count, 1)), "token_accuracy": item_correct / max(count, 1),
        "target_tokens": count, "local_tokens": local, "displaced_tokens": displaced,
        "accessible_tokens": local + displaced, "retrieved_tokens": retrieved,
        "active_tokens": local + retrieved, "active_fraction": (local + retrieved) / max(local + displaced, 1),
        "num_references": len(item.get("references") or []), "num_selected_chunks": len({h.chunk_id for h in hits}),
        "num_selected_references": len(selected), "selected_reference_uris": selected,
        "oracle_selected_reference_uris": sorted(targets), "selection_hit": bool(targets & set(selected)),
        "recall_at_k": len(targets & set(selected)) / max(len(targets), 1),
        "routing_score_statistics": {"count": len(scores), "min": min(scores, default=None),
                                     "max": max(scores, default=None),
                                     "mean": sum(scores) / len(scores) if scores else None},
        "routing_latency": sum(float(d.get("routing_duration_seconds", 0.0)) for d in diag),
        "kv_materialization_latency": sum(float(d.get("materialization_duration_seconds", 0.0)) for d in diag),
        "attention_latency": sum(float(d.get("memory_attention_duration_seconds", 0.0)) for d in diag),
        "kv_transfer_bytes": sum(float(d.get("retrieved_kv_transfer_bytes", 0.0)) for d in diag),
        "example_latency": time.perf_counter() - t_item,
        "search_strategy": cfg.search_strategy, "top_k_references": cfg.top_k_references,
        "top_k_chunks_per_reference": cfg.top_k_chunks_per_reference, "gist_mode": cfg.gist_mode,
        **_complete_reference_rank_metrics(rankings, targets),
    }
