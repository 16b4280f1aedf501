"""Retrieval ranking metrics (``src/pra_torch/metrics.py``)."""

import math

from .runtime.metrics import RunningAverages, ThroughputTimer, cuda_memory_allocated, grad_norm, perplexity


def ranking_metrics(selected: list[str], expected: set[str]) -> dict[str, float]:
    """Binary-relevance hit@1/hit@k/recall/precision/F1/MRR/nDCG over a de-duplicated ranking."""
    ranked = list(dict.fromkeys(selected))
    flags = [item in expected for item in ranked]
    hits = sum(flags)
    mrr = next((1.0 / r for r, f in enumerate(flags, 1) if f), 0.0)
    dcg = sum(1.0 / math.log2(r + 1) for r, f in enumerate(flags, 1) if f)
    ideal = sum(1.0 / math.log2(r + 1) for r in range(1, min(len(expected), len(ranked)) + 1))
    recall, precision = hits / max(len(expected), 1), hits / max(len(ranked), 1)
    return {"hit_at_1": float(bool(flags and flags[0])), "hit_at_k": float(hits > 0), "recall_at_k": recall,
            "precision_at_k": precision, "f1_at_k": 2 * precision * recall / max(precision + recall, 1e-12),
            "mrr": mrr, "ndcg": dcg / max(ideal, 1e-12) if expected else 0.0, "selected_count": float(len(ranked))}


def span_iou(first: tuple[int, int], second: tuple[int, int]) -> float:
    inter = max(min(first[1], second[1]) - max(first[0], second[0]), 0)
    return inter / max(max(first[1], second[1]) - min(first[0], second[0]), 1)


def chunk_is_relevant(hit, target_ids: set[str], target_spans: list[dict], mode: str, iou: float) -> bool:
    if hit.chunk_id in target_ids:
        return True
    mine = (hit.token_start, hit.token_end)
    for span in target_spans:
        if span.get("uri") != hit.source_uri:
            continue
        target = (int(span["token_start"]), int(span["token_end"]))
        if mode == "any_overlap" and min(target[1], mine[1]) > max(target[0], mine[0]):
            return True
        if mode == "iou_threshold" and span_iou(target, mine) >= iou:
            return True
    return False


__all__ = ["RunningAverages", "ThroughputTimer", "chunk_is_relevant", "cuda_memory_allocated", "grad_norm",
           "perplexity", "ranking_metrics", "span_iou"]
