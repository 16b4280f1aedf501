"""Variable-length memory attention: bucket planner and the PyTorch definitions.

``native_kv_attention`` is the canonical transport: one softmax over
``[selected memory (fully visible) ; local keys (causal + padding)]``
(``src/pra_torch/memory_batching.py:216-307``).  ``dynamic_memory_attention``
is the legacy separately-normalised cross-attention, bucketed by similar memory
length with empty rows giving exactly zero (``memory_batching.py:126-213``).

These functions are the readable definitions used on CPU and as the oracle of
the fused ragged kernels in ``pdattention_b200.ops.attention``; unlike the
reference they process the whole batch in one masked program instead of a
per-row Python loop, and keep diagnostics on the device.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class MemoryBucket:
    original_indices: tuple[int, ...]
    lengths: tuple[int, ...]
    max_length: int


@dataclass(frozen=True)
class MemoryBatchingStats:
    selected_lengths: tuple[int, ...]
    requested_bucket_count: int
    actual_bucket_count: int
    bucket_membership: tuple[tuple[int, ...], ...]
    bucket_max_lengths: tuple[int, ...]
    valid_positions: int
    allocated_positions: int
    padding_positions: int
    padding_fraction: float
    attention_entropy: float = 0.0
    attention_max_weight: float = 0.0

    def as_metrics(self) -> dict[str, float]:
        n = max(len(self.selected_lengths), 1)
        return {
            "memory_valid_positions": float(self.valid_positions),
            "memory_allocated_positions": float(self.allocated_positions),
            "memory_padding_positions": float(self.padding_positions),
            "memory_padding_fraction": self.padding_fraction,
            "memory_actual_bucket_count": float(self.actual_bucket_count),
            "memory_max_selected_length": float(max(self.selected_lengths, default=0)),
            "memory_mean_selected_length": float(sum(self.selected_lengths) / n),
            "memory_zero_selection_fraction": float(sum(x == 0 for x in self.selected_lengths) / n),
            "memory_attention_entropy": self.attention_entropy,
            "memory_attention_max_weight": self.attention_max_weight,
        }


class MemoryBucketPlanner:
    """Group similar memory lengths into at most ``max_buckets`` padded rectangles.

    ``optimal_contiguous`` is an exact dynamic program over the length-sorted
    rows minimising allocated positions; ``equal_count`` splits evenly; a zero
    cap isolates every non-empty row.
    """

    def plan(self, lengths: Sequence[int], max_buckets: int, strategy: str = "optimal_contiguous") -> list[MemoryBucket]:
        if max_buckets <= 0:
            return [MemoryBucket((i,), (int(n),), int(n)) for i, n in enumerate(lengths) if n]
        items = sorted(((int(n), i) for i, n in enumerate(lengths) if int(n) > 0))
        if not items:
            return []
        count = min(int(max_buckets), len(items))
        if count == 1:
            groups = [items]
        elif strategy == "equal_count":
            bounds = [k * len(items) // count for k in range(count + 1)]
            groups = [items[a:b] for a, b in zip(bounds, bounds[1:]) if a < b]
        elif strategy == "optimal_contiguous":
            groups = self._optimal_groups(items, count)
        else:
            raise ValueError(f"Unsupported memory bucket strategy: {strategy}")
        return [MemoryBucket(tuple(i for _, i in g), tuple(n for n, _ in g), max(n for n, _ in g)) for g in groups]

    @staticmethod
    def _optimal_groups(items, count):
        n = len(items)
        inf = float("inf")
        best = [[inf] * (n + 1) for _ in range(count + 1)]
        cut = [[-1] * (n + 1) for _ in range(count + 1)]
        best[0][0] = 0
        for k in range(1, count + 1):
            for end in range(k, n + 1):
                width = items[end - 1][0]  # sorted ascending: the group's max
                for start in range(k - 1, end):
                    cost = best[k - 1][start] + (end - start) * width
                    if cost < best[k][end]:
                        best[k][end], cut[k][end] = cost, start
        groups, end = [], n
        for k in range(count, 0, -1):
            start = cut[k][end]
            groups.append(items[start:end])
            end = start
        return groups[::-1]


def _pad_memory(q, memory_k, memory_v):
    lengths = [int(k.shape[2]) for k in memory_k]
    width = max(lengths, default=0)
    b, h, _, dh = q.shape
    keys = q.new_zeros((b, h, width, dh))
    values = q.new_zeros((b, h, width, dh))
    for row, (k, v) in enumerate(zip(memory_k, memory_v)):
        if k.ndim != 4 or v.ndim != 4 or k.shape != v.shape:
            raise ValueError("Each memory K/V pair must have matching [1,H,M,Dh] shapes.")
        if k.shape[0] != 1 or k.shape[1] != h or k.shape[3] != dh:
            raise ValueError("Memory K/V head dimensions do not match the query.")
        keys[row, :, : lengths[row]] = k[0].to(q.device, q.dtype)
        values[row, :, : lengths[row]] = v[0].to(q.device, q.dtype)
    valid = torch.arange(width, device=q.device)[None, :] < torch.tensor(lengths, device=q.device)[:, None]
    return keys, values, valid, lengths


def _weights_stats(weights: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    tiny = torch.finfo(weights.dtype).tiny
    entropy = -(weights * weights.clamp_min(tiny).log()).sum(dim=-1).mean()
    return entropy, weights.max()


def padded_memory_attention(q, memory_k_by_item, memory_v_by_item):
    """Separately normalised attention over one padded rectangle of row memories."""
    if len(memory_k_by_item) != q.shape[0] or len(memory_v_by_item) != q.shape[0]:
        raise ValueError("Memory rows must match the query batch.")
    keys, values, valid, lengths = _pad_memory(q, memory_k_by_item, memory_v_by_item)
    if not lengths or max(lengths) == 0:
        return torch.zeros_like(q), 0.0, 0.0
    scores = (q @ keys.transpose(-2, -1)) / (q.shape[-1] ** 0.5)
    scores = scores.masked_fill(~valid[:, None, None, :], torch.finfo(scores.dtype).min)
    weights = F.softmax(scores, dim=-1) * valid[:, None, None, :]
    entropy, peak = _weights_stats(weights)
    return weights @ values, float(entropy.detach().cpu()), float(peak.detach().cpu())


def dynamic_memory_attention(q, memory_k_by_item, memory_v_by_item, *, bucket_count: int, bucket_strategy: str):
    """Bucketed legacy memory attention; output rows restored to batch order."""
    if len(memory_k_by_item) != q.shape[0] or len(memory_v_by_item) != q.shape[0]:
        raise ValueError("Memory list length must match query batch size.")
    lengths = [int(k.shape[2]) for k in memory_k_by_item]
    buckets = MemoryBucketPlanner().plan(lengths, bucket_count, strategy=bucket_strategy)
    out = torch.zeros_like(q)
    entropies, peaks = [], []
    for bucket in buckets:
        rows = torch.tensor(bucket.original_indices, device=q.device, dtype=torch.long)
        part, entropy, peak = padded_memory_attention(q.index_select(0, rows),
                                                      [memory_k_by_item[i] for i in bucket.original_indices],
                                                      [memory_v_by_item[i] for i in bucket.original_indices])
        out = out.index_copy(0, rows, part)
        entropies.append(entropy)
        peaks.append(peak)
    valid = sum(lengths)
    allocated = sum(len(b.original_indices) * b.max_length for b in buckets)
    stats = MemoryBatchingStats(tuple(lengths), int(bucket_count), len(buckets),
                                tuple(b.original_indices for b in buckets), tuple(b.max_length for b in buckets),
                                valid, allocated, allocated - valid, (allocated - valid) / max(allocated, 1),
                                sum(entropies) / max(len(entropies), 1), sum(peaks) / max(len(peaks), 1))
    return out, stats


def native_kv_attention(q, local_k, local_v, memory_k_by_item, memory_v_by_item, *, attention_mask=None,
                        max_context_tokens: int | None = None, collect_stats: bool = True):
    """One softmax over ``[memory ; local]`` for the whole batch (masked, no row loop).

    ``q``/``local_k``/``local_v`` are ``[B,H,T,Dh]``; memory row ``i`` is
    ``[1,H,M_i,Dh]``.  Memory precedes local keys and is visible to every query;
    local keys keep the causal and padding masks.
    """
    if q.shape != local_k.shape or q.shape != local_v.shape:
        raise ValueError("Local Q/K/V must have matching [B,H,T,Dh] shapes.")
    b, _h, t, _dh = q.shape
    if len(memory_k_by_item) != b or len(memory_v_by_item) != b:
        raise ValueError("Memory list length must match query batch size.")
    if attention_mask is not None and attention_mask.shape != (b, t):
        raise ValueError("attention_mask must match the local [B,T] shape.")
    mem_k, mem_v, mem_valid, lengths = _pad_memory(q, memory_k_by_item, memory_v_by_item)
    if max_context_tokens is not None:
        for m in lengths:
            if m + t > int(max_context_tokens):
                raise ValueError("Native attention context exceeds model_max_context_tokens: "
                                 f"{m} memory + {t} local > {max_context_tokens}.")
    keys = torch.cat((mem_k, local_k), dim=2)
    values = torch.cat((mem_v, local_v), dim=2)
    causal = torch.ones(t, t, dtype=torch.bool, device=q.device).tril()
    local_visible = causal[None].expand(b, t, t)
    if attention_mask is not None:
        local_visible = local_visible & attention_mask.to(q.device, torch.bool)[:, None, :]
    visible = torch.cat((mem_valid[:, None, :].expand(b, t, mem_k.shape[2]), local_visible), dim=2)
    scores = (q @ keys.transpose(-2, -1)) * (q.shape[-1] ** -0.5)
    weights = F.softmax(scores.masked_fill(~visible[:, None], float("-inf")), dim=-1)
    out = weights @ values
    entropy = peak = 0.0
    if collect_stats:
        # Per-row averages, then the mean over rows, as the per-row reference loop reports.
        tiny = torch.finfo(weights.dtype).tiny
        ent_rows = -(weights * weights.clamp_min(tiny).log()).sum(dim=-1).mean(dim=(1, 2))
        peak_rows = weights.amax(dim=(1, 2, 3))
        entropy = float(ent_rows.mean().detach().cpu())
        peak = float(peak_rows.mean().detach().cpu())
    valid = sum(lengths)
    stats = MemoryBatchingStats(tuple(lengths), 0, sum(m > 0 for m in lengths),
                                tuple((i,) for i, m in enumerate(lengths) if m), tuple(m for m in lengths if m),
                                valid, valid, 0, 0.0, entropy, peak)
    return out, stats


__all__ = ["MemoryBatchingStats", "MemoryBucket", "MemoryBucketPlanner", "dynamic_memory_attention",
           "native_kv_attention", "padded_memory_attention"]
