"""PRA adapters for the generic engine: batch step, evaluation, ablations, training entry.

Responsibilities of ``src/pra_torch/pra_train.py``: per batch, build one
row-local cache per row, optionally split long prompts into ``#__head``
references, run ONE batched forward over ``PRABatchedMemoryCache``, compute
cross-entropy with ``ignore_index=0`` and the retrieval / sparsity / recursion
metrics; evaluation writes predictions and JSONL traces.

On a CUDA device with the compiled extension the batch step runs the device
path (``pdattention_b200.models.fastpath.device_batch_step``): all rows'
reference encodes are batched into a few waves, routing and selection stay on
the device, and the selection records needed for metrics are copied once.
"""

from __future__ import annotations

import json
import math
import time
from dataclasses import asdict
from pathlib import Path
from typing import Callable

import torch
import torch.nn.functional as F

from .config import CacheServiceConfig, PRAConfig, ResolverServiceConfig, TrainConfig
from .memory.cache import PRABatchedMemoryCache, PRASimpleMemoryCache
from .memory.prompt import IMPLICIT_PROMPT_HEAD_URI, prepare_prompt_batch_for_pra
from .memory.services import build_cache_from_metadata
from .metrics import chunk_is_relevant, ranking_metrics
from .models.tiny import TinyPRAModel
from .runtime.metrics import RunningAverages, cuda_memory_allocated, perplexity
from .runtime.train import TrainingState, create_training_state, move_batch, train_model

_RANK_CUTOFFS = (1, 2, 4, 8, 16, 32)


def _expected_reference_uris(item: dict) -> set[str]:
    explicit = set(item.get("target_reference_uris") or [])
    if explicit:
        return explicit
    ids = set(item.get("target_reference_ids") or [])
    return {ref.uri for ref in item["references"] if ref.id in ids}


def _chunk_ranking_metrics(selected, item, cfg):
    ids = set(item.get("target_chunk_ids") or [])
    spans = list(item.get("target_chunk_spans") or [])
    if not ids and not spans:
        return None
    flags = [chunk_is_relevant(h, ids, spans, cfg.chunk_match_mode, cfg.chunk_iou_threshold) for h in selected]
    expected = len(ids) or len(spans)
    hits = sum(flags)
    dcg = sum(1.0 / math.log2(r + 1) for r, f in enumerate(flags, 1) if f)
    ideal = sum(1.0 / math.log2(r + 1) for r in range(1, min(expected, len(flags)) + 1))
    recall, precision = hits / max(expected, 1), hits / max(len(flags), 1)
    return {"hit_at_1": float(bool(flags and flags[0])), "hit_at_k": float(hits > 0), "recall_at_k": recall,
            "precision_at_k": precision, "f1_at_k": 2 * precision * recall / max(precision + recall, 1e-12),
            "mrr": next((1.0 / r for r, f in enumerate(flags, 1) if f), 0.0), "ndcg": dcg / max(ideal, 1e-12),
            "selected_count": float(len(selected))}


def _deduplicated_reference_order(selected) -> list[str]:
    ranked = sorted(selected, key=lambda h: (h.reference_rank, h.rank_within_reference))
    return list(dict.fromkeys(h.reference_uri for h in ranked))


def _selections_by_row(by_layer: dict[int, list[list]], batch_size: int) -> list[dict[int, list]]:
    rows = [dict() for _ in range(batch_size)]
    for layer_id, layer_rows in by_layer.items():
        if len(layer_rows) != batch_size:
            raise ValueError(f"Layer {layer_id} returned {len(layer_rows)} selection rows for batch {batch_size}.")
        for r, hits in enumerate(layer_rows):
            rows[r][layer_id] = list(hits)
    return rows


def _complete_reference_rank_metrics(rankings_by_layer, target_uris: set[str]) -> dict:
    """Pre-top-k target ranks per layer, recall@k unions and score margins."""
    per_layer, rr, margins, comparisons = {}, [], [], 0
    union = {k: set() for k in _RANK_CUTOFFS}
    recall = {k: [] for k in _RANK_CUTOFFS}
    for layer_id, rankings in sorted(rankings_by_layer.items()):
        uris = [str(c["reference_uri"]) for c in rankings]
        pos = {u: r for r, u in enumerate(uris, start=1)}
        ranks = sorted(pos[u] for u in target_uris if u in pos)
        rr.append(1.0 / ranks[0] if ranks else 0.0)
        tgt = [float(c["reference_score"]) for c in rankings if c["reference_uri"] in target_uris]
        other = [float(c["reference_score"]) for c in rankings if c["reference_uri"] not in target_uris]
        best_t, best_o = (max(tgt) if tgt else None), (max(other) if other else None)
        margin = best_t - best_o if best_t is not None and best_o is not None else None
        if margin is not None:
            margins.append(margin)
        comparisons += sum(int(ch.get("gist_count", 1)) for c in rankings for ch in c.get("chunks", []))
        row = {"ranked_reference_uris": uris, "target_reference_ranks": ranks, "mrr": rr[-1],
               "best_target_score": best_t, "best_non_target_score": best_o, "score_margin": margin}
        for k in _RANK_CUTOFFS:
            top = set(uris[:k])
            union[k].update(top)
            recall[k].append(len(top & target_uris) / max(len(target_uris), 1))
            row[f"recall_at_{k}"] = recall[k][-1]
        per_layer[str(layer_id)] = row
    out = {"routing_mrr": sum(rr) / max(len(rr), 1),
           "routing_score_margin": sum(margins) / len(margins) if margins else None,
           "gist_comparisons": comparisons, "target_reference_count": len(target_uris),
           "rank_diagnostics_by_layer": per_layer}
    for k in _RANK_CUTOFFS:
        covered = union[k] & target_uris
        out[f"reference_recall_at_{k}"] = sum(recall[k]) / max(len(recall[k]), 1)
        out[f"any_target_hit_at_{k}"] = float(bool(covered))
        out[f"all_targets_hit_at_{k}"] = float(bool(target_uris) and target_uris <= union[k])
        out[f"fraction_targets_covered_at_{k}"] = len(covered) / max(len(target_uris), 1)
    return out


def _row_batching_metrics(layer_diagnostics: dict, row: int) -> dict[str, float]:
    batching = layer_diagnostics.get("batching")
    if batching is None or row >= len(batching.selected_lengths):
        return {}
    valid = int(batching.selected_lengths[row])
    bucket = next((i for i, members in enumerate(batching.bucket_membership) if row in members), None)
    allocated = int(batching.bucket_max_lengths[bucket]) if bucket is not None else 0
    padding = max(allocated - valid, 0)
    return {"memory_valid_positions": float(valid), "memory_allocated_positions": float(allocated),
            "memory_padding_positions": float(padding), "memory_padding_fraction": padding / max(allocated, 1),
            "memory_bucket_index": float(bucket) if bucket is not None else -1.0}


def _retrieval_metrics(caches, selections, metadata, cfg, diagnostics) -> dict[str, float]:
    """Routing quality, sparsity, recursion and batching metrics averaged over (row, layer)."""
    averages = RunningAverages()
    labelled = units = 0
    if not (len(caches) == len(selections) == len(metadata)):
        raise ValueError("Caches, selections, and metadata must align by logical batch row.")
    for row, (cache, by_layer, item) in enumerate(zip(caches, selections, metadata)):
        expected = _expected_reference_uris(item)
        entries = cache.all_entries()
        depth = max((int(e.metadata.get("resolution_depth", 0)) for e in entries), default=0)
        refs_used = max((int(e.metadata.get("resolution_budget_references_used", 0)) for e in entries), default=0)
        toks_used = max((int(e.metadata.get("resolution_budget_tokens_used", 0)) for e in entries), default=0)
        for layer_id, hits in by_layer.items():
            units += 1
            m = {f"retrieval_reference_{k}": v for k, v in
                 ranking_metrics(_deduplicated_reference_order(hits), expected).items()}
            chunk_m = _chunk_ranking_metrics(hits, item, cfg)
            if chunk_m is not None:
                labelled += 1
                m.update({f"retrieval_chunk_{k}": v for k, v in chunk_m.items()})
            counts = cache.layer_counts(layer_id)
            n_refs, n_chunks = len({h.reference_uri for h in hits}), len(hits)
            batching = _row_batching_metrics(diagnostics.get(layer_id, {}), row)
            tokens = int(batching.get("memory_valid_positions", sum(h.selected_token_count for h in hits)))
            scores = [h.chunk_score for h in hits]
            chunk_gists = [int(c.routing_gist.k.shape[0]) for e in entries
                           for c in (e.layer_memory[layer_id].chunks if layer_id in e.layer_memory else [])]
            ref_gists = [int(e.reference_gists_by_layer[layer_id].k.shape[0]) for e in entries
                         if layer_id in e.reference_gists_by_layer]
            win_i = [h.winning_gist_index for h in hits if h.winning_gist_index is not None]
            win_s = [h.winning_gist_score for h in hits if h.winning_gist_score is not None]
            rwin_i = [h.winning_reference_gist_index for h in hits if h.winning_reference_gist_index is not None]
            rwin_s = [h.winning_reference_gist_score for h in hits if h.winning_reference_gist_score is not None]
            m.update({
                "memory_available_reference_count": counts["references"],
                "memory_available_chunk_count": counts["chunks"], "cache_reference_token_count": counts["tokens"],
                "retrieval_selected_reference_count": n_refs, "retrieval_selected_chunk_count": n_chunks,
                "memory_selected_token_count": tokens,
                "memory_selected_reference_fraction": n_refs / max(counts["references"], 1),
                "memory_selected_chunk_fraction": n_chunks / max(counts["chunks"], 1),
                "memory_selected_token_fraction": tokens / max(counts["tokens"], 1),
                "retrieval_routing_score_mean": sum(scores) / max(len(scores), 1),
                "retrieval_routing_score_max": max(scores, default=0.0),
                "retrieval_zero_chunk_fraction": float(n_chunks == 0),
                "chunk_gists_requested": cfg.gists_per_chunk,
                "chunk_gists_actual_mean": sum(chunk_gists) / max(len(chunk_gists), 1),
                "chunk_gists_actual_max": max(chunk_gists, default=0),
                "reference_gists_requested": cfg.reference_gists_per_reference,
                "reference_gists_actual_mean": sum(ref_gists) / max(len(ref_gists), 1),
                "reference_gists_actual_max": max(ref_gists, default=0),
                "winning_chunk_gist_index": sum(win_i) / max(len(win_i), 1),
                "winning_reference_gist_index": sum(rwin_i) / max(len(rwin_i), 1),
                "chunk_best_gist_score": sum(win_s) / max(len(win_s), 1),
                "reference_best_gist_score": sum(rwin_s) / max(len(rwin_s), 1),
                "memory_retrieved_chunk_attended_fraction": float(tokens > 0) if n_chunks else 0.0,
                "cache_recursive_expansion_depth": depth,
                "cache_recursive_reference_budget_fraction": refs_used / max(cfg.recursive_max_total_references, 1),
                "cache_recursive_token_budget_fraction": toks_used / max(cfg.recursive_max_total_tokens, 1),
            })
            averages.update(m)
            averages.update({f"layer_{layer_id}_{k.removeprefix('retrieval_')}": v for k, v in m.items()})
    for layer_id, diag in diagnostics.items():
        scalars = {k: v for k, v in diag.items() if isinstance(v, (int, float))}
        averages.update(scalars)
        averages.update({f"layer_{layer_id}_{k}": v for k, v in scalars.items()})
    out = averages.compute()
    out["retrieval_chunk_labels_available_fraction"] = labelled / max(units, 1)
    out["reference_retrieval_accuracy"] = out.get("retrieval_reference_hit_at_k", 0.0)
    out["reference_selection_top1_accuracy"] = out.get("retrieval_reference_hit_at_1", 0.0)
    out["reference_selection_topk_accuracy"] = out.get("retrieval_reference_hit_at_k", 0.0)
    out["reference_selection_mrr"] = out.get("retrieval_reference_mrr", 0.0)
    out["selected_ref_count"] = out.get("retrieval_reference_selected_count", 0.0)
    return out


def _sync(device: str) -> None:
    if str(device).startswith("cuda") and torch.cuda.is_available():
        torch.cuda.synchronize()


def _use_device_path(model, device: str) -> bool:
    return str(device).startswith("cuda") and getattr(model, "device_path_enabled", lambda: False)()


def _pra_batch_step(model, batch: dict, device: str, tokenizer, resolver_config: ResolverServiceConfig,
                    cache_config: CacheServiceConfig) -> tuple[torch.Tensor, dict]:
    """Build row-local caches, then ONE batched prompt forward over ``PRABatchedMemoryCache``."""
    if _use_device_path(model, device):
        from .models.fastpath import device_batch_step

        return device_batch_step(model, batch, device, tokenizer, resolver_config, cache_config)
    batch = move_batch(batch, device)
    caches, build_s = [], 0.0
    for item in batch["metadata"]:
        t0 = time.perf_counter()
        caches.append(build_cache_from_metadata(model, tokenizer, [item], device, resolver_config=resolver_config,
                                                cache_config=cache_config, attach_to_model=False))
        build_s += time.perf_counter() - t0
    prepared = None
    if model.cfg.prompt_overflow_mode != "truncate" or model.cfg.max_prompt_direct_tokens is not None:
        t0 = time.perf_counter()
        prepared = prepare_prompt_batch_for_pra(model, tokenizer, batch["input_ids"],
                                                attention_mask=batch.get("attention_mask"),
                                                labels=batch.get("labels"), metadata=batch.get("metadata"),
                                                caches=caches)
        build_s += time.perf_counter() - t0
        batch = {**batch, "input_ids": prepared.input_ids, "attention_mask": prepared.attention_mask,
                 "labels": prepared.labels}
    batch_cache = PRABatchedMemoryCache(caches)
    model.set_pra_cache(batch_cache)
    _sync(device)
    t0 = time.perf_counter()
    logits = model(batch["input_ids"], attention_mask=prepared.attention_mask if prepared is not None else None,
                   position_offset=prepared.position_offsets if prepared is not None else 0)
    _sync(device)
    forward_s = time.perf_counter() - t0
    b = int(batch["input_ids"].shape[0])
    selections = _selections_by_row(model.selected_chunks_by_layer(), b)
    diagnostics = model.pra_diagnostics_by_layer()
    loss = F.cross_entropy(logits.view(-1, logits.size(-1)), batch["labels"].view(-1), ignore_index=0)
    metrics = _retrieval_metrics(caches, selections, batch["metadata"], model.cfg, diagnostics)
    metrics.update({"cache_build_duration_seconds": build_s / max(len(caches), 1),
                    "cache_build_total_duration_seconds": build_s, "logical_batch_size": float(b),
                    "prompt_forward_calls": 1.0, "prompt_forward_duration_seconds": forward_s})
    if prepared is not None:
        _prompt_metrics(metrics, prepared, selections)
    return loss, {"tokens": int(batch["attention_mask"].sum().item()), "examples": b, "batch": batch,
                  "cache": caches[-1] if caches else None, "caches": caches, "batch_cache": batch_cache,
                  "selections": selections, "diagnostics": diagnostics, "metrics": metrics, "logits": logits}


def _prompt_metrics(metrics: dict, prepared, selections) -> None:
    names = tuple(prepared.stats[0].as_metrics()) if prepared.stats else ()
    for name in names:
        metrics[name] = sum(s.as_metrics()[name] for s in prepared.stats) / max(len(prepared.stats), 1)
    per_row = [sum(1 for hits in row.values() for h in hits if h.reference_uri == IMPLICIT_PROMPT_HEAD_URI)
               for row in selections]
    metrics["prompt_implicit_chunks_selected"] = sum(per_row) / max(len(per_row), 1)


def _trace(item, prediction, cache, layer_selections, diagnostics, index, tokenizer, cfg) -> dict:
    events = getattr(cache, "resolution_events", [])
    return {
        "question": item["question"], "answer": item["answer"], "predicted_answer": prediction,
        "available_references": [asdict(ref) for ref in item["references"]],
        "cached_references": list(cache.entries.keys()),
        "selected_references_by_layer": {str(l): _deduplicated_reference_order(s) for l, s in layer_selections.items()},
        "selected_chunks_by_layer": {str(l): [h.as_trace_dict() for h in s] for l, s in layer_selections.items()},
        "expanded_anchors": item.get("expected_anchors", []),
        "expansion_depth": max((e.depth for e in events), default=0),
        "cache_hits": (not _expected_reference_uris(item)
                       or bool(_expected_reference_uris(item).intersection(cache.entries))),
        "retrieved_token_counts": [len(tokenizer.encode(e.text)) for e in cache.all_entries()],
        "memory_lengths_by_layer": {
            str(l): int(_row_batching_metrics(diagnostics.get(l, {}), index).get(
                "memory_valid_positions", sum(h.selected_token_count for h in s)))
            for l, s in layer_selections.items()},
        "bucket_stats_by_layer": {str(l): _row_batching_metrics(d, index) for l, d in diagnostics.items()},
        "recursive_paths": [asdict(e) for e in events],
        "routing_configuration": {"search_strategy": cfg.search_strategy, "top_k_references": cfg.top_k_references,
                                  "top_k_chunks_per_reference": cfg.top_k_chunks_per_reference,
                                  "gist_mode": cfg.gist_mode, "chunking_mode": cfg.chunking_mode,
                                  "detail_materialization": cfg.detail_materialization},
    }


def evaluate_pra_model(*, model: TinyPRAModel, loader, tokenizer, train_config: TrainConfig, device: str, split: str,
                       resolver_config=None, cache_config=None, save_predictions=None, save_traces=None) -> dict:
    """Loss, answer accuracy, routing quality, recursion cost and throughput (+ optional JSONL)."""
    resolver_config = ResolverServiceConfig.from_value(resolver_config or train_config.resolver_config)
    cache_config = CacheServiceConfig.from_value(cache_config or train_config.cache_config)
    was_training = model.training
    model.eval()
    averages = RunningAverages()
    exact = anchor_hits = cache_hits = total = retrieved = expanded = depth = token_total = 0
    t0 = time.perf_counter()
    pred_path, trace_path = (Path(save_predictions) if save_predictions else None,
                             Path(save_traces) if save_traces else None)
    for p in (pred_path, trace_path):
        if p:
            p.parent.mkdir(parents=True, exist_ok=True)
    pred_f = pred_path.open("w", encoding="utf-8") if pred_path else None
    trace_f = trace_path.open("w", encoding="utf-8") if trace_path else None
    try:
        with torch.no_grad():
            for batch in loader:
                loss, out = _pra_batch_step(model, batch, device, tokenizer, resolver_config, cache_config)
                predicted = out["logits"].argmax(dim=-1).detach().cpu()
                averages.update({f"{split}_loss": float(loss.detach().cpu()), **out.get("metrics", {})},
                                weight=max(int(out["examples"]), 1))
                token_total += int(out["tokens"])
                for i, item in enumerate(out["batch"]["metadata"]):
                    cache = out["caches"][i]
                    retrieved += sum(len(tokenizer.encode(e.text)) for e in cache.all_entries())
                    expanded += len(cache.entries)
                    prediction = tokenizer.decode(predicted[i])
                    total += 1
                    exact += int(item["answer"].strip() in prediction)
                    expected = _expected_reference_uris(item)
                    cache_hits += int(not expected or bool(expected.intersection(cache.entries)))
                    events = getattr(cache, "resolution_events", [])
                    depth += max((e.depth for e in events), default=0)
                    anchors = item.get("expected_anchors", [])
                    text = "\n".join(e.text for e in cache.all_entries())
                    anchor_hits += int(not anchors or any(a in text or a in " ".join(cache.entries) for a in anchors))
                    if pred_f:
                        pred_f.write(json.dumps({"id": item["id"], "prediction": prediction,
                                                 "answer": item["answer"]}) + "\n")
                    if trace_f:
                        trace_f.write(json.dumps(_trace(item, prediction, cache, out["selections"][i],
                                                        out["diagnostics"], i, tokenizer, model.cfg),
                                                 default=str) + "\n")
    finally:
        for f in (pred_f, trace_f):
            if f:
                f.close()
        if was_training:
            model.train()
    elapsed = max(time.perf_counter() - t0, 1e-9)
    metrics = averages.compute()
    loss = metrics.get(f"{split}_loss", 0.0)
    metrics.update({"loss": loss, "perplexity": perplexity(loss), "answer_accuracy": exact / max(total, 1),
                    "expected_anchor_hit": anchor_hits / max(total, 1), "expansion_depth": depth / max(total, 1),
                    "expanded_ref_count": expanded / max(total, 1),
                    "average_retrieved_tokens": retrieved / max(total, 1), "cache_hit_ratio": cache_hits / max(total, 1),
                    "latency": elapsed, "examples_per_second": total / elapsed,
                    "tokens_per_second": token_total / elapsed, "gpu_memory_allocated": cuda_memory_allocated(device)})
    return metrics


def native_kv_gap_metrics(results: list[dict]) -> dict[str, float]:
    from .native_metrics import derive_native_kv_metrics

    losses = {str(r["condition"]): float(r["loss"]) for r in results}
    for src, dst in (("valid", "native_routed"), ("native_disabled", "native_disabled")):
        if src in losses:
            losses[dst] = losses[src]
    return derive_native_kv_metrics(losses)


def _pra_checkpoint_extra(cfg: PRAConfig, train_config: TrainConfig, tokenizer, resolver_config, cache_config
                          ) -> Callable[[], dict]:
    return lambda: {
        "cfg": cfg.__dict__, "stoi": tokenizer.stoi, "itos": tokenizer.itos,
        "dataset_stage": train_config.dataset_stage, "resolver_config": resolver_config.__dict__,
        "cache_config": cache_config.__dict__,
        "reference_vocabulary": {k: v for k, v in tokenizer.stoi.items() if str(k).startswith("<REF_")},
        "tokenizer_type": type(tokenizer).__name__,
        "tokenizer_json": tokenizer.to_json() if hasattr(tokenizer, "to_json") else None,
    }


def create_pra_training_state(cfg: PRAConfig, train_config: TrainConfig, datamodule, *, model=None) -> TrainingState:
    model = model or TinyPRAModel(cfg)
    resolver = ResolverServiceConfig.from_value(train_config.resolver_config)
    cache = CacheServiceConfig.from_value(train_config.cache_config)
    return create_training_state(model, train_config, checkpoint_extra=_pra_checkpoint_extra(
        cfg, train_config, datamodule.tokenizer, resolver, cache))


def train_pra_model(*, cfg: PRAConfig, train_config: TrainConfig, datamodule, model=None, resolver_config=None,
                    cache_config=None, state: TrainingState | None = None):
    """Bind the PRA batch / eval steps to the generic engine."""
    tokenizer = datamodule.tokenizer
    resolver_config = ResolverServiceConfig.from_value(resolver_config or train_config.resolver_config)
    cache_config = CacheServiceConfig.from_value(cache_config or train_config.cache_config)
    extra = _pra_checkpoint_extra(cfg, train_config, tokenizer, resolver_config, cache_config)
    if state is None:
        state = create_training_state(model or TinyPRAModel(cfg), train_config, checkpoint_extra=extra)
    else:
        state.checkpoint_extra = extra

    def batch_step(current, batch, device):
        return _pra_batch_step(current, batch, device, tokenizer, resolver_config, cache_config)

    def eval_step(current, loader, device, split="val"):
        return evaluate_pra_model(model=current, loader=loader, tokenizer=tokenizer, train_config=train_config,
                                  device=device, split=split, resolver_config=resolver_config,
                                  cache_config=cache_config)

    return train_model(model=state.model, train_config=train_config, train_loader=datamodule.train_loader(),
                       val_loader=datamodule.val_loader(), test_loader=datamodule.test_loader(),
                       batch_step=batch_step, eval_step=eval_step, state=state)


def training_step(model, batch: dict, device: str, tokenizer, optimizer, *, resolver_config=None, cache_config=None,
                  scheduler=None, max_grad_norm: float = 1.0, next_batch: dict | None = None) -> tuple[torch.Tensor, dict]:
    """One optimizer step on one batch: cache build, routed forward, loss, backward, clip, update.

    This is the unit the training engine repeats; it is public so drivers and
    benchmarks run exactly the code path users get.  Returns ``(loss, info)``
    with the loss still on the device (read it when needed).  With ``next_batch``
    a device-path model plans that batch's cache build on the host while this
    step's kernels run.
    """
    resolver_config = ResolverServiceConfig.from_value(resolver_config)
    cache_config = CacheServiceConfig.from_value(cache_config)
    optimizer.zero_grad(set_to_none=True)
    announce = getattr(model, "announce_batch", None)
    if next_batch is not None and announce is not None:
        announce(next_batch)
    loss, info = _pra_batch_step(model, batch, device, tokenizer, resolver_config, cache_config)
    loss.backward()
    hook = getattr(model, "optimizer_step_hook", None)
    if hook is not None:
        hook(optimizer, type("Cfg", (), {"max_grad_norm": max_grad_norm})())
    else:
        if max_grad_norm:
            torch.nn.utils.clip_grad_norm_(model.parameters(), max_grad_norm)
        optimizer.step()
    if scheduler is not None:
        scheduler.step()
    prefetch = getattr(model, "prefetch_batch", None)
    if next_batch is not None and prefetch is not None:
        prefetch(next_batch)
    return loss, info


from .ablation import evaluate_reference_ablation  # noqa: E402  (re-export, keeps the reference import path)
