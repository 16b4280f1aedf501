"""TinyGPT-PRA: decoder-only LM plus the reference-cache encoder.

Architecture and state-dict layout of ``src/pra_torch/model.py:31-1305``:
learned absolute positions, a vanilla prefix (``nn.TransformerEncoderLayer``
layout, pre-norm, GELU), mixed blocks (vanilla MHA + PRA + MLP with Dropout at
``ff.2``), then PRA blocks (``ln1 -> PRAttention -> ln2 -> MLP``), a final
LayerNorm and an untied bias-free head.  Reference chunk K/V is projected from
the same normalised state the PRA sublayer consumes.

Execution on CUDA goes through ``pdattention_b200.models.fastpath`` (bf16
sm_100a kernels, batched multi-row cache build).  The methods here are the
reference-semantics object path used on CPU, by the generic cache API and as
the numerical oracle.
"""

from __future__ import annotations

from contextlib import nullcontext
from dataclasses import replace
import warnings

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..chunking import partition_reference_tokens, partition_source
from ..config import PRAConfig
from ..memory.cache import (
    ChunkRoutingGist,
    LayerKV,
    LayerReferenceMemory,
    PRACacheEntry,
    PRAMemoryCache,
    PRASimpleMemoryCache,
    ReferenceChunkMemory,
    ReferenceRoutingGists,
)
from ..memory.gists import GRUGistPooler, GistContext, compute_gists, projected_tokens
from .attention import PRAttention


def causal_attention_mask(seq_len: int, device) -> torch.Tensor:
    """``[T,T]`` boolean mask, true above the diagonal (hidden future keys)."""
    return torch.ones(seq_len, seq_len, dtype=torch.bool, device=device).triu(1)


def _mha(attn: nn.MultiheadAttention, x, causal: bool, attention_mask=None):
    """Self-attention with an ``nn.MultiheadAttention`` parameter layout."""
    t = x.shape[1]
    mask = causal_attention_mask(t, x.device) if causal else None
    padding = ~attention_mask.bool() if attention_mask is not None else None
    out, _ = attn(x, x, x, attn_mask=mask, key_padding_mask=padding, need_weights=False)
    return out


class _EncoderLayer(nn.Module):
    """Parameter container with the ``nn.TransformerEncoderLayer`` names."""

    def __init__(self, cfg: PRAConfig):
        super().__init__()
        self.self_attn = nn.MultiheadAttention(cfg.d_model, cfg.n_heads, dropout=cfg.dropout, batch_first=True)
        self.linear1 = nn.Linear(cfg.d_model, cfg.d_ff)
        self.dropout = nn.Dropout(cfg.dropout)
        self.linear2 = nn.Linear(cfg.d_ff, cfg.d_model)
        self.norm1 = nn.LayerNorm(cfg.d_model)
        self.norm2 = nn.LayerNorm(cfg.d_model)
        self.dropout1 = nn.Dropout(cfg.dropout)
        self.dropout2 = nn.Dropout(cfg.dropout)

    def forward(self, x, attention_mask=None):
        x = x + self.dropout1(_mha(self.self_attn, self.norm1(x), True, attention_mask))
        return x + self.dropout2(self.linear2(self.dropout(F.gelu(self.linear1(self.norm2(x))))))


class VanillaTransformerBlock(nn.Module):
    """Causal pre-norm block with no memory branch."""

    def __init__(self, cfg: PRAConfig, layer_id: int):
        super().__init__()
        self.layer_id = layer_id
        self.layer = _EncoderLayer(cfg)

    def forward(self, x, use_pra_memory: bool = True, attention_mask=None):
        del use_pra_memory
        return self.layer(x, attention_mask)


class PRATransformerBlock(nn.Module):
    """``x + attn(ln1(x))`` then ``x + ff(ln2(x))``."""

    def __init__(self, cfg: PRAConfig, layer_id: int, pra_cache: PRAMemoryCache):
        super().__init__()
        self.layer_id = layer_id
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.attn = PRAttention(cfg.d_model, cfg.n_heads, cfg.max_seq_len, layer_id, pra_cache, config=cfg)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.ff = nn.Sequential(nn.Linear(cfg.d_model, cfg.d_ff), nn.GELU(), nn.Linear(cfg.d_ff, cfg.d_model))

    def forward(self, x, use_pra_memory: bool = True, attention_mask=None):
        x = x + self.attn(self.ln1(x), use_pra_memory=use_pra_memory, attention_mask=attention_mask)
        return x + self.ff(self.ln2(x))

    def set_pra_cache(self, pra_cache: PRAMemoryCache) -> None:
        self.attn.pra_cache = pra_cache

    def project_reference_kv(self, x, *, detach: bool = True):
        return self.attn.project_kv(self.ln1(x), detach=detach)

    @property
    def pra_layer(self) -> PRAttention:
        return self.attn


class PRASATransformerBlock(nn.Module):
    """Vanilla causal MHA residual, then a PRA residual, then the MLP."""

    def __init__(self, cfg: PRAConfig, layer_id: int, pra_cache: PRAMemoryCache):
        super().__init__()
        self.layer_id = layer_id
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.self_attn = nn.MultiheadAttention(cfg.d_model, cfg.n_heads, dropout=cfg.dropout, batch_first=True)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.pra_attn = PRAttention(cfg.d_model, cfg.n_heads, cfg.max_seq_len, layer_id, pra_cache, config=cfg)
        self.ln3 = nn.LayerNorm(cfg.d_model)
        self.ff = nn.Sequential(nn.Linear(cfg.d_model, cfg.d_ff), nn.GELU(), nn.Dropout(cfg.dropout),
                                nn.Linear(cfg.d_ff, cfg.d_model))

    def _apply_self_attention(self, x, attention_mask=None):
        return x + _mha(self.self_attn, self.ln1(x), True, attention_mask)

    def forward(self, x, use_pra_memory: bool = True, attention_mask=None):
        x = self._apply_self_attention(x, attention_mask)
        x = x + self.pra_attn(self.ln2(x), use_pra_memory=use_pra_memory, attention_mask=attention_mask)
        return x + self.ff(self.ln3(x))

    def set_pra_cache(self, pra_cache: PRAMemoryCache) -> None:
        self.pra_attn.pra_cache = pra_cache

    def project_reference_kv(self, x, *, detach: bool = True):
        return self.pra_attn.project_kv(self.ln2(self._apply_self_attention(x)), detach=detach)

    @property
    def pra_layer(self) -> PRAttention:
        return self.pra_attn


def _pra_layer(block) -> PRAttention | None:
    return getattr(block, "pra_layer", None)


class TinyPRAModel(nn.Module):
    """Decoder-only LM whose blocks also encode references into layer caches."""

    def __init__(self, cfg: PRAConfig, pra_cache: PRAMemoryCache | None = None):
        super().__init__()
        self.cfg = cfg
        self.pra_cache = pra_cache if pra_cache is not None else PRASimpleMemoryCache()
        self.token_emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.pos_emb = nn.Embedding(cfg.max_seq_len, cfg.d_model)
        modes = {cfg.gist_mode, cfg.reference_level_gist_mode}
        needs_gru = "gru" in modes or ("hybrid" in modes and cfg.gist_hybrid_global_mode == "gru")
        self.gist_pooler = (GRUGistPooler(cfg.d_model, hidden_size=cfg.gist_gru_hidden_size,
                                          num_layers=cfg.gist_gru_num_layers,
                                          bidirectional=cfg.gist_gru_bidirectional, dropout=cfg.dropout)
                            if needs_gru else None)
        self.blocks = nn.ModuleList(self._build_blocks(cfg))
        self.ln = nn.LayerNorm(cfg.d_model)
        self.head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        self.last_generation_stats: dict = {}

    def _build_blocks(self, cfg: PRAConfig) -> list[nn.Module]:
        blocks = []
        for layer_id in range(cfg.n_layers):
            if layer_id < cfg.n_vanilla_layers:
                blocks.append(VanillaTransformerBlock(cfg, layer_id))
            elif layer_id < cfg.n_vanilla_layers + cfg.n_mixed_layers:
                blocks.append(PRASATransformerBlock(cfg, layer_id, self.pra_cache))
            else:
                blocks.append(PRATransformerBlock(cfg, layer_id, self.pra_cache))
        return blocks

    # -- cache binding and traces ------------------------------------------
    def pra_layers(self) -> list[PRAttention]:
        return [layer for layer in map(_pra_layer, self.blocks) if layer is not None]

    def set_pra_cache(self, pra_cache: PRAMemoryCache) -> None:
        self.pra_cache = pra_cache
        for block in self.blocks:
            if hasattr(block, "set_pra_cache"):
                block.set_pra_cache(pra_cache)

    def clear_pra_cache(self) -> None:
        self.pra_cache.clear()

    def selected_chunks_by_layer(self) -> dict[int, list[list]]:
        return {layer.layer_id: [list(row) for row in layer.last_selected_chunks] for layer in self.pra_layers()}

    def routing_rankings_by_layer(self) -> dict[int, list[list[dict]]]:
        return {layer.layer_id: [list(row) for row in layer.last_routing_rankings] for layer in self.pra_layers()}

    def selected_references_by_layer(self) -> dict[int, list[list[tuple[str, float]]]]:
        warnings.warn("selected_references_by_layer() is deprecated; use selected_chunks_by_layer().",
                      DeprecationWarning, stacklevel=2)
        out = {}
        for layer_id, rows in self.selected_chunks_by_layer().items():
            out[layer_id] = []
            for hits in rows:
                first = {}
                for h in hits:
                    first.setdefault(h.reference_uri, h.reference_score)
                out[layer_id].append(list(first.items()))
        return out

    def pra_diagnostics_by_layer(self) -> dict[int, dict]:
        return {layer.layer_id: {**layer.last_diagnostics, "batching": layer.last_memory_batching_stats}
                for layer in self.pra_layers()}

    # -- language-model forward ------------------------------------------------
    def positions(self, b: int, t: int, device, attention_mask=None, position_offset=0) -> torch.Tensor:
        """Positional embeddings ``[B or 1, T, D]`` with range checks on the native limit."""
        limit = self.cfg.effective_model_max_context_tokens
        if torch.is_tensor(position_offset):
            offsets = position_offset.to(device=device, dtype=torch.long).reshape(-1)
            if offsets.numel() != b:
                raise ValueError("Per-row position offsets must have shape [batch].")
            pos = offsets[:, None] + torch.arange(t, device=device)[None, :]
            valid = attention_mask.bool() if attention_mask is not None else torch.ones_like(pos, dtype=torch.bool)
            used = pos[valid]
            if used.numel() and (int(used.min()) < 0 or int(used.max()) >= limit):
                raise ValueError("Prompt positions exceed the model positional table.")
            return self.pos_emb(pos.masked_fill(~valid, 0))
        offset = int(position_offset)
        if offset < 0 or offset + t > limit:
            raise ValueError("Prompt position range exceeds the model positional table: "
                             f"[{offset}, {offset + t}) vs model_max_context_tokens={limit}.")
        return self.pos_emb(torch.arange(offset, offset + t, device=device))[None]

    def forward(self, input_ids, use_pra_memory: bool = True, attention_mask=None,
                position_offset: int | torch.Tensor = 0):
        b, t = input_ids.shape
        limit = self.cfg.effective_model_max_context_tokens
        if t > limit:
            raise ValueError(f"Native forward has {t} tokens, exceeding model_max_context_tokens={limit}.")
        if attention_mask is not None and attention_mask.shape != input_ids.shape:
            raise ValueError("attention_mask must have the same [batch,tokens] shape as input_ids.")
        x = self.token_emb(input_ids) + self.positions(b, t, input_ids.device, attention_mask, position_offset)
        for block in self.blocks:
            x = block(x, use_pra_memory=use_pra_memory, attention_mask=attention_mask)
        return self.head(self.ln(x))

    # -- reference encoding (object path) -------------------------------------
    def _encode_reference_tokens(self, token_ids, device, *, detach: bool, use_pra_memory: bool,
                                 position_offset: int = 0) -> dict[int, LayerKV]:
        """Run one source independently; capture ``[1,H,M,Dh]`` K/V before each PRA sublayer."""
        ids = torch.tensor([list(token_ids)], dtype=torch.long, device=device)
        limit = self.cfg.effective_model_max_context_tokens
        offset = int(position_offset)
        if ids.shape[1] > limit:
            raise ValueError(f"Reference encoding call has {ids.shape[1]} tokens, exceeding "
                             f"model_max_context_tokens={limit}.")
        if offset < 0 or offset + ids.shape[1] > limit:
            raise ValueError("Reference position range exceeds the model positional table: "
                             f"[{offset}, {offset + ids.shape[1]}) vs model_max_context_tokens={limit}.")
        x = self.token_emb(ids) + self.pos_emb(torch.arange(offset, offset + ids.shape[1], device=device))[None]
        captured = {}
        for block in self.blocks:
            if hasattr(block, "project_reference_kv"):
                captured[block.layer_id] = block.project_reference_kv(x, detach=detach)
            x = block(x, use_pra_memory=use_pra_memory)
        return captured

    def _cache_resident_kv(self, kv: LayerKV) -> LayerKV:
        if self.cfg.kv_cache_residency == "gpu":
            return kv
        k, v = kv.k.detach().to("cpu"), kv.v.detach().to("cpu")
        if self.cfg.kv_cache_pin_memory and torch.cuda.is_available():
            k, v = k.pin_memory(), v.pin_memory()
        return LayerKV(k, v)

    def _gists(self, kv: LayerKV, token_ids, tokenizer, detach: bool, summary_k=None, summary_available=False):
        computed = compute_gists(
            keys=projected_tokens(kv.k), values=projected_tokens(kv.v), mode=self.cfg.gist_mode,
            num_gists=self.cfg.gists_per_chunk, config=self.cfg,
            context=GistContext(level="chunk", token_ids=token_ids, tokenizer=tokenizer,
                                ref_end_token=self.cfg.ref_end_token, gru_pooler=self.gist_pooler))
        k, v = computed.k, computed.v
        if detach:
            k, v = k.detach(), (v.detach() if v is not None else None)
        return ChunkRoutingGist(k=k, v=v, method=self.cfg.gist_mode, summary_k=summary_k,
                                metadata={**computed.metadata, "summary_available": summary_available})

    def _reference_gists(self, memory: LayerReferenceMemory, detach: bool) -> ReferenceRoutingGists:
        keys = torch.cat([c.routing_gist.k for c in memory.chunks], dim=0)
        has_v = all(c.routing_gist.v is not None for c in memory.chunks)
        values = torch.cat([c.routing_gist.v for c in memory.chunks], dim=0) if has_v else None
        computed = compute_gists(keys=keys, values=values, mode=self.cfg.reference_level_gist_mode,
                                 num_gists=self.cfg.reference_gists_per_reference, config=self.cfg,
                                 context=GistContext(level="reference", gru_pooler=self.gist_pooler))
        k, v = computed.k, computed.v
        if detach:
            k, v = k.detach(), (v.detach() if v is not None else None)
        return ReferenceRoutingGists(k=k, v=v, mode=self.cfg.reference_level_gist_mode, metadata=computed.metadata)

    def rebuild_cache_routing_gists(self, cache: PRAMemoryCache | None = None, *, tokenizer=None) -> None:
        """Re-pool routing gists from stored K/V under the current gist settings (no re-encode)."""
        cache = cache or self.pra_cache
        detach = self.cfg.cache_build_mode == "detached"
        with torch.no_grad() if detach else nullcontext():
            for entry in cache.all_entries():
                for layer_id, memory in entry.layer_memory.items():
                    for chunk in memory.chunks:
                        ids = tuple(chunk.metadata.get("source_token_ids") or ())
                        old = chunk.routing_gist
                        chunk.routing_gist = self._gists(chunk.token_kv, ids, tokenizer, detach, old.summary_k,
                                                         old.summary_k is not None)
                    if self.cfg.reference_level_gist_mode is None or not memory.chunks:
                        entry.reference_gists_by_layer.pop(layer_id, None)
                        continue
                    entry.reference_gists_by_layer[layer_id] = self._reference_gists(memory, detach)
                entry.metadata.update({"gist_mode": self.cfg.gist_mode, "gists_per_chunk": self.cfg.gists_per_chunk,
                                       "reference_level_gist_mode": self.cfg.reference_level_gist_mode,
                                       "reference_gists_per_reference": self.cfg.reference_gists_per_reference})
        if hasattr(cache, "invalidate_routing_indexes"):
            cache.invalidate_routing_indexes()

    def _bounded_reference_payloads(self, uri, token_ids, tokenizer, device, metadata, *, detach, use_pra_memory,
                                    historical_encoding, max_chunks, use_configured_max_chunks):
        """Encode model-safe blocks (optional left context) and slice K/V into routing chunks."""
        cfg = self.cfg
        limit = cfg.effective_model_max_context_tokens
        encoding = cfg.encoding_chunking_config
        cores = partition_source(uri, token_ids, tokenizer, replace(encoding, overlap_fraction=0.0, overlap_tokens=0),
                                 {**metadata, "partition_level": "encoding"}, max_chunks=None,
                                 overflow_policy="error", max_chunk_tokens=limit)
        mode = ("historical_window" if historical_encoding and cfg.encoding_context_mode == "independent"
                else cfg.encoding_context_mode)
        payloads, widest, total = [], 0, 0
        for block_index, core in enumerate(cores):
            core_ids = list(core.token_ids)
            want = encoding.resolved_overlap_tokens(len(core_ids)) if mode in {"overlap", "historical_window"} else 0
            left = min(core.token_start, want, max(limit - len(core_ids), 0))
            start = core.token_start - left
            encode_ids = list(token_ids[start: core.token_end])
            widest, total = max(widest, len(encode_ids)), total + len(encode_ids)
            offset = start if cfg.reference_position_mode == "global" and start + len(encode_ids) <= limit else 0
            encoded = self._encode_reference_tokens(encode_ids, device, detach=detach,
                                                    use_pra_memory=use_pra_memory and not historical_encoding,
                                                    position_offset=offset)
            core_kv = {lid: LayerKV(kv.k[:, :, left: left + len(core_ids)], kv.v[:, :, left: left + len(core_ids)])
                       for lid, kv in encoded.items()}
            for local in partition_source(uri, core_ids, tokenizer, cfg.routing_chunking_config,
                                          {**metadata, "partition_level": "routing"}, max_chunks=None,
                                          overflow_policy="error", max_chunk_tokens=limit):
                g0, g1 = core.token_start + local.token_start, core.token_start + local.token_end
                routed = replace(local, chunk_id=f"{uri}#chunk={len(payloads)}", token_start=g0, token_end=g1,
                                 metadata={**local.metadata, "encoding_block_id": block_index,
                                           "encoding_input_start": start, "encoding_input_end": core.token_end,
                                           "encoding_input_tokens": len(encode_ids), "encoding_context_tokens": left,
                                           "logical_start_token": g0, "logical_end_token": g1,
                                           "base_model_position_offset": offset})
                payloads.append((routed, {lid: LayerKV(kv.k[:, :, local.token_start: local.token_end],
                                                       kv.v[:, :, local.token_start: local.token_end])
                                          for lid, kv in core_kv.items()}))
        cap = cfg.max_gists_per_reference if use_configured_max_chunks else max_chunks
        dropped = max(len(payloads) - cap, 0) if cap is not None else 0
        if dropped:
            if cfg.gist_overflow_policy == "error":
                raise ValueError(f"Reference produced {len(payloads)} routing chunks, exceeding {cap}.")
            payloads = payloads[:cap]
        routing = cfg.routing_chunking_config
        return payloads, {
            "encoding_call_count": len(cores), "max_encoding_input_tokens": widest,
            "encoding_input_tokens_total": total, "encoding_context_mode": mode,
            "encoding_chunking": {"mode": encoding.mode, "chunk_tokens": encoding.chunk_tokens,
                                  "overlap_tokens": encoding.overlap_tokens,
                                  "overlap_fraction": encoding.overlap_fraction},
            "routing_chunking": {"mode": routing.mode, "chunk_tokens": routing.chunk_tokens,
                                 "overlap_tokens": routing.overlap_tokens, "overlap_fraction": routing.overlap_fraction},
            "discarded_chunk_count": dropped,
        }

    def encode_reference_to_cache(self, uri: str, text: str, tokenizer, device, metadata: dict | None = None, *,
                                  use_pra_memory: bool = False) -> PRACacheEntry:
        return self.encode_reference_tokens_to_cache(uri, tokenizer.encode(text), tokenizer, device, metadata,
                                                     text=text, use_pra_memory=use_pra_memory)

    def entry_metadata(self, metadata: dict, chunks, token_ids, historical_encoding, bounded, stats) -> dict:
        cfg = self.cfg
        encoded = sum(len(c.token_ids) for c in chunks)
        return {
            **metadata, "chunking_mode": cfg.routing_chunking_config.mode, "gist_mode": cfg.gist_mode,
            "gists_per_chunk": cfg.gists_per_chunk, "reference_level_gist_mode": cfg.reference_level_gist_mode,
            "reference_gists_per_reference": cfg.reference_gists_per_reference,
            "cache_build_mode": cfg.cache_build_mode, "use_summary": cfg.use_summary, "summary_mode": cfg.summary_mode,
            "chunk_count": len(chunks), "chunk_overlap_fraction": cfg.chunk_overlap_fraction,
            "chunk_overlap_tokens": cfg.resolved_chunk_overlap_tokens,
            "overlap_materialization": cfg.overlap_materialization, "historical_encoding": bool(historical_encoding),
            "reference_encoding_strategy": "bounded_native_slice" if bounded else "independent",
            "model_max_context_tokens": cfg.effective_model_max_context_tokens,
            "logical_context_tokens": len(token_ids),
            "logical_to_native_context_ratio": len(token_ids) / max(cfg.effective_model_max_context_tokens, 1),
            **stats, "unique_source_tokens": len(token_ids), "encoded_tokens_including_overlap": encoded,
            "duplication_factor": encoded / max(len(token_ids), 1),
        }

    def encode_reference_tokens_to_cache(self, uri: str, token_ids, tokenizer, device, metadata: dict | None = None, *,
                                         text: str | None = None, use_pra_memory: bool = False,
                                         max_chunks: int | None = None, use_configured_max_chunks: bool = True,
                                         max_chunk_tokens: int | None = None,
                                         historical_encoding: bool = False) -> PRACacheEntry:
        """Partition exact ids and build per-layer chunk K/V plus gists (not yet published)."""
        cfg = self.cfg
        metadata = dict(metadata or {})
        token_ids = [int(t) for t in token_ids]
        text = tokenizer.decode(token_ids) if text is None else text
        detach = cfg.cache_build_mode == "detached"
        grad_mode = torch.no_grad() if detach else nullcontext()
        limit = cfg.effective_model_max_context_tokens
        bounded = historical_encoding or cfg.encoding_chunking is not None or len(token_ids) > limit
        pre_encoded = {}
        if bounded:
            if use_pra_memory and historical_encoding:
                raise ValueError("Historical source encoding cannot consume its own PRA memory.")
            with grad_mode:
                payloads, stats = self._bounded_reference_payloads(
                    uri, token_ids, tokenizer, device, metadata, detach=detach, use_pra_memory=use_pra_memory,
                    historical_encoding=historical_encoding, max_chunks=max_chunks,
                    use_configured_max_chunks=use_configured_max_chunks)
            chunks = [c for c, _ in payloads]
            pre_encoded = {c.chunk_id: kv for c, kv in payloads}
        else:
            chunks = partition_reference_tokens(uri, token_ids, tokenizer, cfg, metadata, text=text,
                                                max_chunks=max_chunks,
                                                use_configured_max_chunks=use_configured_max_chunks,
                                                max_chunk_tokens=max_chunk_tokens or limit)
            stats = {"encoding_call_count": len(chunks),
                     "max_encoding_input_tokens": max((len(c.token_ids) for c in chunks), default=0),
                     "encoding_input_tokens_total": sum(len(c.token_ids) for c in chunks),
                     "encoding_context_mode": "independent"}
        entry = PRACacheEntry(uri=uri, text=text, child_uris=list(metadata.get("child_uris") or []),
                              metadata=self.entry_metadata(metadata, chunks, token_ids, historical_encoding, bounded,
                                                           stats))
        with grad_mode:
            summary_by_layer = self._summary_gists(metadata.get("summary"), tokenizer, device, detach)
            for chunk in chunks:
                ids = list(chunk.token_ids)
                original = len(ids)
                if original > limit:
                    if cfg.reference_overflow_policy == "error":
                        raise ValueError(f"Chunk {chunk.chunk_id} has {original} tokens, exceeding "
                                         f"model_max_context_tokens={limit}.")
                    ids = ids[:limit]
                layer_kv = pre_encoded.get(chunk.chunk_id)
                if layer_kv is None:
                    layer_kv = self._encode_reference_tokens(ids, device, detach=detach, use_pra_memory=use_pra_memory)
                for layer_id, kv in layer_kv.items():
                    gist = self._gists(kv, ids, tokenizer, detach, summary_by_layer.get(layer_id),
                                       layer_id in summary_by_layer)
                    memory = ReferenceChunkMemory(
                        chunk_id=chunk.chunk_id, source_uri=chunk.source_uri, token_start=chunk.token_start,
                        token_end=min(chunk.token_start + len(ids), chunk.token_end), char_start=chunk.char_start,
                        char_end=chunk.char_end, token_kv=self._cache_resident_kv(kv), routing_gist=gist,
                        metadata={**chunk.metadata, "source_token_ids": tuple(ids), "original_token_count": original,
                                  "retained_token_count": len(ids), "truncated": original != len(ids)})
                    entry.layer_memory.setdefault(layer_id, LayerReferenceMemory()).chunks.append(memory)
            if cfg.reference_level_gist_mode is not None:
                for layer_id, memory in entry.layer_memory.items():
                    if memory.chunks:
                        entry.reference_gists_by_layer[layer_id] = self._reference_gists(memory, detach)
        return entry

    def _summary_gists(self, summary, tokenizer, device, detach) -> dict:
        cfg = self.cfg
        if not (cfg.use_summary and summary):
            return {}
        ids = list(tokenizer.encode(str(summary)))[: cfg.effective_model_max_context_tokens]
        if not ids:
            return {}
        mode = "gru" if cfg.gist_mode == "gru" else "mean"
        out = {}
        for layer_id, kv in self._encode_reference_tokens(ids, device, detach=detach, use_pra_memory=False).items():
            out[layer_id] = compute_gists(
                keys=projected_tokens(kv.k), values=None, num_gists=1, config=cfg, mode=mode,
                context=GistContext(level="chunk", token_ids=ids, tokenizer=tokenizer,
                                    ref_end_token=cfg.ref_end_token, gru_pooler=self.gist_pooler)).k
        return out

    def encode_reference_group_to_cache(self, references: list[dict], tokenizer, device) -> list[PRACacheEntry]:
        """Contextualise consecutive URIs jointly (``block_slice`` / ``native_slice``) and slice back by URI."""
        cfg = self.cfg
        if cfg.reference_encoding_strategy == "independent":
            raise ValueError("Grouped encoding requires block_slice or native_slice.")
        if cfg.use_summary:
            raise NotImplementedError("Grouped reference encoding does not yet support summaries.")
        rows, flat, starts = [], [], []
        for ref in references:
            ids = tuple(int(t) for t in tokenizer.encode(str(ref["text"])))
            if ids:
                starts.append(len(flat))
                flat.extend(ids)
                rows.append({**ref, "token_ids": ids})
        if not rows:
            return []
        starts.append(len(flat))
        size = len(rows) if cfg.reference_encoding_strategy == "native_slice" else cfg.encoding_block_references
        limit = cfg.effective_model_max_context_tokens
        blocks, encoded_total = [], 0
        for block_id, r0 in enumerate(range(0, len(rows), size)):
            r1 = min(r0 + size, len(rows))
            c0, c1 = starts[r0], starts[r1]
            want = max(1, int((c1 - c0) * cfg.encoding_overlap_fraction)) if cfg.encoding_overlap_fraction > 0 else 0
            overlap = min(c0, want)
            ids = flat[c0 - overlap: c1]
            if len(ids) > limit:
                raise ValueError(f"Encoding block {block_id} has {len(ids)} tokens, exceeding "
                                 f"model_max_context_tokens={limit}.")
            encoded_total += len(ids)
            blocks.append({"block_id": block_id, "row_start": r0, "row_end": r1, "encode_start": c0 - overlap,
                           "core_start": c0, "core_end": c1, "overlap_tokens": overlap, "encode_ids": ids})
        run_id = (f"{rows[0]['uri']}|{cfg.reference_encoding_strategy}|{cfg.encoding_block_references}|"
                  f"{cfg.encoding_overlap_fraction}|{cfg.reference_position_mode}")
        common = {"encoding_run_id": run_id, "reference_encoding_strategy": cfg.reference_encoding_strategy,
                  "encoding_block_references": cfg.encoding_block_references,
                  "encoding_overlap_fraction": cfg.encoding_overlap_fraction,
                  "reference_position_mode": cfg.reference_position_mode,
                  "encoding_run_unique_source_tokens": len(flat),
                  "encoding_run_encoded_tokens_including_overlap": encoded_total,
                  "encoding_run_stored_kv_tokens": len(flat),
                  "encoding_run_duplication_factor": encoded_total / max(len(flat), 1)}
        entries = {str(r["uri"]): PRACacheEntry(uri=str(r["uri"]), text=str(r["text"]), metadata={
            **dict(r.get("metadata") or {}), **common, "chunking_mode": "grouped_uri_slice",
            "gist_mode": cfg.gist_mode, "gists_per_chunk": cfg.gists_per_chunk,
            "unique_source_tokens": len(r["token_ids"]), "encoded_tokens_including_overlap": len(r["token_ids"]),
            "stored_kv_tokens_including_overlap": len(r["token_ids"])}) for r in rows}
        detach = cfg.cache_build_mode == "detached"
        with torch.no_grad() if detach else nullcontext():
            for block in blocks:
                start = block["encode_start"]
                offset = start if cfg.reference_position_mode == "global" and start + len(block["encode_ids"]) <= limit else 0
                layer_kv = self._encode_reference_tokens(block["encode_ids"], device, detach=detach,
                                                         use_pra_memory=False, position_offset=offset)
                for r in range(block["row_start"], block["row_end"]):
                    row = rows[r]
                    a, z = starts[r] - start, starts[r + 1] - start
                    entry = entries[str(row["uri"])]
                    for layer_id, kv in layer_kv.items():
                        part = LayerKV(kv.k[:, :, a:z], kv.v[:, :, a:z])
                        chunk = ReferenceChunkMemory(
                            chunk_id=f"{row['uri']}#chunk=0", source_uri=str(row["uri"]), token_start=0,
                            token_end=len(row["token_ids"]), token_kv=self._cache_resident_kv(part),
                            routing_gist=self._gists(part, row["token_ids"], tokenizer, detach),
                            metadata={"source_token_ids": row["token_ids"], "encoding_block_id": block["block_id"],
                                      "encoding_block_core_tokens": block["core_end"] - block["core_start"],
                                      "encoding_overlap_tokens": block["overlap_tokens"],
                                      "global_token_start": starts[r], "global_token_end": starts[r + 1]})
                        chunk.routing_gist.metadata.pop("summary_available", None)
                        entry.layer_memory.setdefault(layer_id, LayerReferenceMemory()).chunks.append(chunk)
        if cfg.reference_level_gist_mode is not None:
            temporary = PRASimpleMemoryCache()
            for entry in entries.values():
                temporary.put(entry)
            self.rebuild_cache_routing_gists(temporary, tokenizer=tokenizer)
        return [entries[str(r["uri"])] for r in rows]

    # -- generation -------------------------------------------------------------
    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens=64, temperature=1.0, use_pra_memory: bool = True, *,
                 tokenizer=None, do_sample: bool = True):
        """Autoregressive generation with streaming ``#__head`` rollover."""
        from .generation import generate_with_rollover

        return generate_with_rollover(self, input_ids, max_new_tokens, temperature, use_pra_memory,
                                      tokenizer=tokenizer, do_sample=do_sample)


TinyPRALanguageModel = TinyPRAModel
TransformerBlock = PRATransformerBlock


def convert_sa_model_to_pra(source: TinyPRAModel, target_config: PRAConfig, *,
                            pra_cache: PRAMemoryCache | None = None) -> TinyPRAModel:
    """Copy a ``td_sa`` model into a native-KV PRA architecture (exact with memory disabled)."""
    if source.cfg.model_variant != "td_sa":
        raise ValueError("Source model must use model_variant='td_sa'.")
    if target_config.memory_transport != "native_kv":
        raise ValueError("SA conversion targets canonical memory_transport='native_kv'.")
    fields = ("vocab_size", "d_model", "n_heads", "n_layers", "d_ff", "max_seq_len")
    differ = [f for f in fields if getattr(source.cfg, f) != getattr(target_config, f)]
    if differ:
        raise ValueError(f"Source and target architecture differ in: {', '.join(differ)}")
    target = TinyPRAModel(target_config, pra_cache=pra_cache)
    with torch.no_grad():
        for name in ("token_emb", "pos_emb", "ln", "head"):
            getattr(target, name).load_state_dict(getattr(source, name).state_dict())
        for src, dst in zip(source.blocks, target.blocks):
            if not isinstance(src, VanillaTransformerBlock):
                raise TypeError("Every source td_sa block must be vanilla self-attention.")
            if isinstance(dst, VanillaTransformerBlock):
                dst.load_state_dict(src.state_dict())
                continue
            if not isinstance(dst, PRATransformerBlock):
                raise TypeError("SA conversion supports vanilla or PRA target blocks.")
            layer = src.layer
            dst.ln1.load_state_dict(layer.norm1.state_dict())
            dst.ln2.load_state_dict(layer.norm2.state_dict())
            weights = layer.self_attn.in_proj_weight.chunk(3, dim=0)
            biases = layer.self_attn.in_proj_bias.chunk(3, dim=0)
            for proj, w, b in zip((dst.attn.q_proj, dst.attn.k_proj, dst.attn.v_proj), weights, biases):
                proj.weight.copy_(w)
                proj.bias.copy_(b)
            dst.attn.o_proj.load_state_dict(layer.self_attn.out_proj.state_dict())
            dst.ff[0].load_state_dict(layer.linear1.state_dict())
            dst.ff[2].load_state_dict(layer.linear2.state_dict())
    return target


def convert_sa_checkpoint_to_pra(checkpoint: dict, target_config: PRAConfig, *,
                                 map_location: str | torch.device = "cpu") -> TinyPRAModel:
    values = dict(checkpoint["cfg"])
    values["device"] = str(map_location)
    source = TinyPRAModel(PRAConfig(**values)).to(map_location)
    source.load_state_dict(checkpoint["model"])
    return convert_sa_model_to_pra(source, target_config).to(map_location)
