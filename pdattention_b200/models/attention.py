"""PRA attention: causal local attention plus routed native-K/V memory.

Behaviour of ``src/pra_torch/attention.py:27-628``:

1. local causal multi-head attention over ``q,k,v = split(q/k/v_proj(x))``;
2. the routing query is the last *valid* token's ``q`` flattened to ``[B,D]``;
3. the cache routes every row in its own namespace;
4. per row: optional ``full_reference`` expansion, ``chunk_score >=
   trigger_threshold``, ``(uri, chunk_id)`` de-duplication, a greedy whole-chunk
   budget in ``(-score, uri, chunk_id)`` order under ``model_max_context - T -
   reserve`` (capped by ``max_materialized_memory_tokens``; cost 1 per chunk in
   ``gist_only`` mode), then spans sorted by ``(uri, token_start, chunk_id)``
   with overlap already covered by the same URI stripped;
5. ``native_kv``: one softmax over ``[memory ; local]`` and the ordinary
   ``o_proj``; ``cross_attention``: separately normalised, bucketed memory
   attention through ``mem_o_proj`` added as ``local + alpha * memory``.

Two execution paths share these semantics:

* the *object path* (this module) -- host-side selection over
  ``SelectedChunk`` records; used on CPU, for traces and as the oracle;
* the *device path* (``pdattention_b200.models.fastpath``) -- fused sm_100a
  routing + selection + ragged attention kernels with no host round trip,
  taken when a compiled ``DeviceMemoryPlan`` is attached to the layer.
"""

from __future__ import annotations

import math
import time
from dataclasses import replace

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..memory.batching import MemoryBatchingStats, dynamic_memory_attention, native_kv_attention
from ..memory.cache import LayerKV, PRAMemoryCache, SelectedChunk

_BUDGET_SUM_KEYS = ("direct_context_tokens", "memory_budget_tokens", "routing_candidates", "routing_topk_candidates",
                    "chunks_materialized", "chunks_budget_rejected", "memory_tokens_requested",
                    "memory_tokens_materialized")


def _fence(tensor: torch.Tensor, enabled: bool) -> None:
    if enabled and tensor.is_cuda:
        torch.cuda.synchronize(tensor.device)


def budget_selection(selected: list[SelectedChunk], config, *, direct_tokens: int, routing_candidates: int):
    """Greedy whole-chunk budget in ``(-score, uri, chunk_id)`` order (skip what does not fit)."""
    hard = config.effective_model_max_context_tokens - int(direct_tokens) - config.context_safety_reserve_tokens
    if hard < 0:
        raise ValueError("Direct context and safety reserve exceed model_max_context_tokens.")
    budget = hard if config.max_materialized_memory_tokens is None else min(hard, config.max_materialized_memory_tokens)
    gist_only = config.detail_materialization == "gist_only"
    ranked = sorted(selected, key=lambda h: (-h.chunk_score, h.reference_uri, h.chunk_id))
    cost = [1 if gist_only else h.selected_token_count for h in ranked]
    kept, rejected, left = [], [], budget
    for hit, c in zip(ranked, cost):
        if c <= left:
            kept.append(hit)
            left -= c
        else:
            rejected.append(hit)
    used = budget - left
    return kept, {
        "model_max_context_tokens": float(config.effective_model_max_context_tokens),
        "direct_context_tokens": float(direct_tokens),
        "memory_budget_tokens": float(budget),
        "routing_candidates": float(routing_candidates),
        "routing_topk_candidates": float(len(selected)),
        "chunks_materialized": float(len(kept)),
        "chunks_budget_rejected": float(len(rejected)),
        "memory_tokens_requested": float(sum(cost)),
        "memory_tokens_materialized": float(used),
        "materialization_budget_utilization": used / max(budget, 1),
        "lowest_materialized_score": min((h.chunk_score for h in kept), default=float("nan")),
        "highest_budget_rejected_score": max((h.chunk_score for h in rejected), default=float("nan")),
    }


class PRAttention(nn.Module):
    """Causal attention with routed memory (parameter layout of the reference)."""

    def __init__(self, d_model, n_heads, max_seq_len, layer_id, pra_cache: PRAMemoryCache, *, config):
        super().__init__()
        if d_model % n_heads:
            raise ValueError("d_model must be divisible by n_heads.")
        self.d_model, self.n_heads, self.head_dim = d_model, n_heads, d_model // n_heads
        self.max_seq_len, self.layer_id, self.config = max_seq_len, layer_id, config
        self.trigger_threshold = config.trigger_threshold
        self.memory_transport = config.memory_transport
        self.memory_alpha = config.memory_alpha
        self.pra_cache = pra_cache
        self.last_selected_chunks: list[list[SelectedChunk]] = []
        self.last_routing_rankings: list[list[dict]] = []
        self.last_memory_batching_stats: MemoryBatchingStats | None = None
        self.last_diagnostics: dict[str, float] = {}
        self.device_plan = None  # compiled DeviceMemoryPlan for the fused path
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.o_proj = nn.Linear(d_model, d_model)
        self.mem_o_proj = nn.Linear(d_model, d_model) if self.memory_transport == "cross_attention" else None
        self.register_buffer("causal_mask", torch.tril(torch.ones(max_seq_len, max_seq_len)).view(
            1, 1, max_seq_len, max_seq_len))

    # -- shapes ------------------------------------------------------------
    def split_heads(self, x):
        b, t, _ = x.shape
        return x.view(b, t, self.n_heads, self.head_dim).transpose(1, 2)

    def merge_heads(self, x):
        b, h, t, d = x.shape
        return x.transpose(1, 2).contiguous().view(b, t, h * d)

    def project_kv(self, hidden_states, *, detach: bool = True) -> LayerKV:
        """``[1,M,D]`` normalised states -> this layer's ``[1,H,M,Dh]`` cache K/V."""
        k = self.split_heads(self.k_proj(hidden_states))
        v = self.split_heads(self.v_proj(hidden_states))
        return LayerKV(k.detach(), v.detach()) if detach else LayerKV(k, v)

    def forward_native_kv(self, x, memory_k, memory_v, *, attention_mask=None):
        """Native attention with caller-supplied historical K/V (routing bypassed)."""
        if self.memory_transport != "native_kv":
            raise RuntimeError("forward_native_kv requires memory_transport='native_kv'.")
        q, k, v = (self.split_heads(p(x)) for p in (self.q_proj, self.k_proj, self.v_proj))
        heads, _ = native_kv_attention(q, k, v, memory_k, memory_v, attention_mask=attention_mask,
                                       max_context_tokens=self.config.effective_model_max_context_tokens)
        return self.o_proj(self.merge_heads(heads))

    # -- selection -----------------------------------------------------------
    def _expand_full_references(self, selected):
        out, seen = [], set()
        for hit in selected:
            if hit.reference_uri in seen:
                continue
            seen.add(hit.reference_uri)
            memory = hit.entry.layer_memory.get(self.layer_id)
            if memory is None:
                continue
            for rank, chunk in enumerate(memory.chunks, start=1):
                out.append(replace(hit, chunk=chunk, rank_within_reference=rank,
                                   metadata={**hit.metadata, "materialization": "full_reference"}))
        return out

    def _budget_selection(self, selected, *, direct_tokens: int, routing_candidates: int):
        return budget_selection(selected, self.config, direct_tokens=direct_tokens,
                                routing_candidates=routing_candidates)

    def _materialize(self, selected, q, *, direct_tokens: int):
        """One row's hits -> ``[1,H,M,Dh]`` K/V (+ retained hits, overlap, transfer stats)."""
        cfg = self.config
        candidates = len(selected)
        if cfg.detail_materialization == "full_reference":
            selected = self._expand_full_references(selected)
        selected = [h for h in selected if h.chunk_score >= self.trigger_threshold]
        unique, seen = [], set()
        for h in selected:
            key = (h.reference_uri, h.chunk_id)
            if key not in seen:
                seen.add(key)
                unique.append(h)
        selected, stats = self._budget_selection(unique, direct_tokens=direct_tokens, routing_candidates=candidates)
        empty = q.new_empty((1, self.n_heads, 0, self.head_dim))
        if not selected:
            return empty, empty, selected, 0, 0, 0.0, stats
        keys, values, duplicates, covered = [], [], 0, {}
        for h in sorted(selected, key=lambda s: (s.reference_uri, s.token_start, s.chunk_id)):
            if cfg.detail_materialization == "gist_only":
                gist = h.chunk.routing_gist
                w = 0 if h.winning_gist_index is None else int(h.winning_gist_index)
                w = min(max(w, 0), max(int(gist.k.shape[0]) - 1, 0))
                kv = gist.k[w]
                vv = gist.v[w] if gist.v is not None else kv
                key, value = kv.view(1, self.n_heads, 1, self.head_dim), vv.view(1, self.n_heads, 1, self.head_dim)
            else:
                key, value = h.chunk.token_kv.k, h.chunk.token_kv.v
                end = covered.get(h.reference_uri, h.token_start)
                overlap = min(max(end - h.token_start, 0), int(key.shape[2]))
                if overlap:
                    duplicates += overlap
                    if cfg.overlap_materialization == "deduplicate":
                        key, value = key[:, :, overlap:], value[:, :, overlap:]
                covered[h.reference_uri] = max(end, h.token_end)
            if key.shape[2]:
                keys.append(key)
                values.append(value)
        if not keys:
            return empty, empty, selected, duplicates, 0, 0.0, stats
        moved = sum(k.numel() * k.element_size() + v.numel() * v.element_size()
                    for k, v in zip(keys, values) if k.device != q.device or v.device != q.device)
        timing = cfg.collect_detailed_timing and moved > 0
        _fence(q, timing)
        start = time.perf_counter()
        keys = [k.to(q.device, q.dtype, non_blocking=cfg.kv_cache_non_blocking) for k in keys]
        values = [v.to(q.device, q.dtype, non_blocking=cfg.kv_cache_non_blocking) for v in values]
        _fence(q, timing)
        elapsed = time.perf_counter() - start if moved else 0.0
        return torch.cat(keys, dim=2), torch.cat(values, dim=2), selected, duplicates, moved, elapsed, stats

    # -- forward -------------------------------------------------------------
    def _local_attention(self, q, k, v, attention_mask):
        b, _, t, _ = q.shape
        scores = q @ k.transpose(-2, -1) / math.sqrt(self.head_dim)
        scores = scores.masked_fill(self.causal_mask[:, :, :t, :t] == 0, float("-inf"))
        if attention_mask is not None:
            if attention_mask.shape != (b, t):
                raise ValueError(f"Expected attention_mask {(b, t)}, got {tuple(attention_mask.shape)}.")
            valid = attention_mask.to(device=q.device, dtype=torch.bool)
            if not bool(valid.any(dim=1).all()):
                raise ValueError("Every prompt row must contain at least one direct token.")
            scores = scores.masked_fill(~valid[:, None, None, :], float("-inf"))
        return F.softmax(scores, dim=-1) @ v

    @staticmethod
    def routing_query(q: torch.Tensor, attention_mask) -> torch.Tensor:
        """Last valid token's ``q`` per row, flattened to ``[B,D]``."""
        b, h, t, dh = q.shape
        if attention_mask is None:
            picked = q[:, :, -1, :]
        else:
            pos = torch.arange(t, device=q.device).expand(b, -1)
            last = pos.masked_fill(~attention_mask.bool(), -1).max(dim=1).values
            picked = q.gather(2, last.view(b, 1, 1, 1).expand(-1, h, 1, dh)).squeeze(2)
        return picked.contiguous().view(b, h * dh)

    def forward(self, x, use_pra_memory: bool = True, attention_mask: torch.Tensor | None = None):
        if self.device_plan is not None and use_pra_memory:
            from .fastpath import pra_attention_device

            return pra_attention_device(self, x, attention_mask)
        b, t, _ = x.shape
        self.last_selected_chunks = [[] for _ in range(b)]
        self.last_routing_rankings = [[] for _ in range(b)]
        self.last_memory_batching_stats = None
        self.last_diagnostics = {}
        q, k, v = (self.split_heads(p(x)) for p in (self.q_proj, self.k_proj, self.v_proj))
        local_out = self.o_proj(self.merge_heads(self._local_attention(q, k, v, attention_mask)))
        if not use_pra_memory or self.pra_cache.is_empty():
            return local_out

        cfg = self.config
        timing = cfg.collect_detailed_timing
        query = self.routing_query(q, attention_mask)
        _fence(q, timing)
        t0 = time.perf_counter()
        selected_rows = self.pra_cache.search(query, self.layer_id, cfg)
        if hasattr(self.pra_cache, "last_rankings"):
            self.last_routing_rankings = self.pra_cache.last_rankings(self.layer_id)
        _fence(q, timing)
        routing_s = time.perf_counter() - t0

        _fence(q, timing)
        t0 = time.perf_counter()
        mem_k, mem_v, budgets = [], [], []
        duplicates = moved = 0
        transfer_s = 0.0
        for row, selected in enumerate(selected_rows):
            key, value, kept, dup, row_moved, row_s, row_stats = self._materialize(selected, q[row:row + 1],
                                                                                   direct_tokens=t)
            mem_k.append(key)
            mem_v.append(value)
            self.last_selected_chunks[row] = kept
            duplicates += dup
            moved += row_moved
            transfer_s += row_s
            budgets.append(row_stats)
        _fence(q, timing)
        materialize_s = time.perf_counter() - t0
        summed = {key: sum(float(r[key]) for r in budgets) for key in _BUDGET_SUM_KEYS}
        shared = {
            "model_max_context_tokens": float(cfg.effective_model_max_context_tokens),
            **summed,
            "direct_context_tokens": float(t * b),
            "materialization_budget_utilization": sum(r["materialization_budget_utilization"] for r in budgets)
            / max(len(budgets), 1),
            "memory_duplicate_chunk_tokens": float(duplicates),
            "retrieved_kv_transfer_bytes": float(moved),
        }
        timings = {"routing_duration_seconds": routing_s, "materialization_duration_seconds": materialize_s,
                   "selected_kv_transfer_duration_seconds": transfer_s}

        if self.memory_transport == "native_kv":
            if not any(int(kk.shape[2]) for kk in mem_k):
                self.last_diagnostics = {k_: sum(float(r[k_]) for r in budgets) for k_ in _BUDGET_SUM_KEYS}
                self.last_diagnostics["model_max_context_tokens"] = float(cfg.effective_model_max_context_tokens)
                return local_out
            _fence(q, timing)
            t0 = time.perf_counter()
            heads, stats = native_kv_attention(q, k, v, mem_k, mem_v, attention_mask=attention_mask,
                                               max_context_tokens=cfg.effective_model_max_context_tokens)
            _fence(q, timing)
            timings["memory_attention_duration_seconds"] = time.perf_counter() - t0
            self.last_memory_batching_stats = stats
            output = self.o_proj(self.merge_heads(heads))
            self.last_diagnostics = native_diagnostics(self, stats, shared, budgets, output, local_out,
                                                       attention_mask, duplicates, q, b, t)
            if timing:
                self.last_diagnostics.update(timings)
            return output

        _fence(q, timing)
        t0 = time.perf_counter()
        mem_heads, stats = dynamic_memory_attention(q, mem_k, mem_v, bucket_count=cfg.memory_bucket_count,
                                                    bucket_strategy=cfg.memory_bucket_strategy)
        _fence(q, timing)
        timings["memory_attention_duration_seconds"] = time.perf_counter() - t0
        self.last_memory_batching_stats = stats
        memory_out = self.mem_o_proj(self.merge_heads(mem_heads))
        has_memory = torch.tensor([n > 0 for n in stats.selected_lengths], device=memory_out.device,
                                  dtype=memory_out.dtype).view(b, 1, 1)
        memory_out = memory_out * has_memory
        mem_norm = float(memory_out.detach().norm().cpu())
        loc_norm = float(local_out.detach().norm().cpu())
        self.last_diagnostics = {**stats.as_metrics(), **shared, "memory_output_norm": mem_norm,
                                 "local_output_norm": loc_norm,
                                 "memory_to_local_output_norm_ratio": mem_norm / max(loc_norm, 1e-12)}
        if timing:
            self.last_diagnostics.update(timings)
        return local_out + self.memory_alpha * memory_out


def native_diagnostics(layer, stats, shared, budgets, output, local_out, attention_mask, duplicates, q, b, t) -> dict:
    cfg = layer.config
    local_tokens = int(attention_mask.sum().item()) if attention_mask is not None else b * t
    retrieved = int(stats.valid_positions)
    dedup = cfg.overlap_materialization == "deduplicate"
    accessible = local_tokens + retrieved
    out_norm = float(output.detach().norm().cpu())
    loc_norm = float(local_out.detach().norm().cpu())
    finite = [r["lowest_materialized_score"] for r in budgets if math.isfinite(r["lowest_materialized_score"])]
    rejected = [r["highest_budget_rejected_score"] for r in budgets
                if math.isfinite(r["highest_budget_rejected_score"])]
    return {
        **stats.as_metrics(), **shared,
        "lowest_materialized_score": min(finite, default=float("nan")),
        "highest_budget_rejected_score": max(rejected, default=float("nan")),
        "memory_transport_native_kv": 1.0,
        "active_local_tokens": float(local_tokens),
        "retrieved_token_kv": float(retrieved),
        "retrieved_physical_kv_tokens": float(retrieved),
        "retrieved_unique_source_tokens": float(retrieved if dedup else max(retrieved - duplicates, 0)),
        "selected_stored_kv_tokens": float(retrieved + duplicates if dedup else retrieved),
        "memory_overlap_tokens_detected": float(duplicates),
        "memory_overlap_tokens_removed": float(duplicates if dedup else 0),
        "accessible_kv_tokens": float(accessible),
        "active_memory_fraction": retrieved / max(accessible, 1),
        "retrieved_kv_storage_bytes": float(2 * retrieved * layer.n_heads * layer.head_dim * q.element_size()),
        "attention_output_norm": out_norm,
        "local_output_norm": loc_norm,
        "attention_to_local_output_norm_ratio": out_norm / max(loc_norm, 1e-12),
    }
