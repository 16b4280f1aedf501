"""Device execution path of TinyGPT-PRA on B200 (bf16 sm_100a kernels).

What changes relative to the object path (same semantics, different execution):

* **Parameters** live in flat buffers: fp32 masters (the ``nn.Parameter``
  storage, so ``state_dict`` keeps the reference layout), a bf16 compute copy,
  a bf16 gradient buffer written directly by the weight-gradient GEMMs, and the
  AdamW moments; one fused kernel clips and updates everything.
* **Cache build** for a whole batch: every row's recursive build plan is traced
  on the host by the native planner (``pra_ops.plan_batch``, ``csrc/planner.cpp``;
  the Python planner ``plan_cache_builds`` is its oracle and fallback), entries
  are grouped into *waves* by their
  visibility dependencies (an encode that reads memory runs after everything it
  can see), and each wave encodes all its chunks of all rows in ONE batched
  forward.  The QKV GEMM of every layer writes straight into a per-layer pool,
  which IS the chunk K/V store (zero copy); gists (mean or k-means) are pooled
  on the device from those rows.
* **Routing + selection + materialisation** run in one kernel per layer
  (``pra_ops.route``) against row-local namespaces, producing the memory key
  list consumed by the ragged attention kernel -- no host round trip.

Unsupported configurations (legacy cross-attention transport, reference-first
or global-chunks search, summaries, trainable gists, grouped encoding, CPU
residency, head widths other than 32/64/128) keep using the object path.
"""

from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from ..chunking import partition_reference_tokens
from ..memory.gists import kmeanspp_random_stream
from ..memory.gists.strategies import local_generator
from ..config import ResolverServiceConfig
from ..memory.services import plan_cache_builds
from ..ops import _ext
from ..tracing import nvtx_range, traced
from ..ops.kernels import (DropoutStreams, MemoryView, WeightSlot, attention, dropout_add, layer_norm, linear,
                           lm_head_loss, lm_head_logits, mlp)
from .native_plan import NativeBatchPlan, native_config
from .tiny import PRATransformerBlock, TinyPRAModel

_AGG = {"max": 0, "mean": 1, "logsumexp": 2}
_ALIGN = 8  # elements: every flat region starts 16-byte aligned (TMA and vector loads need 16)


def _upload(device, *arrays, dtype=torch.int32) -> list[torch.Tensor]:
    """Copy several host integer sequences to the device in ONE asynchronous copy.

    The sequences are packed into a pinned staging buffer, so the copy neither
    blocks the host nor synchronises the stream (a pageable ``torch.tensor(...,
    device=cuda)`` does both); the returned tensors are views of one device
    buffer.  Empty sequences come back as a one-element zero tensor.
    """
    import numpy as np

    parts = [np.asarray(a if len(a) else [0], dtype=np.int64 if dtype == torch.int64 else np.int32).ravel()
             for a in arrays]
    sizes = [p.size for p in parts]
    host = torch.from_numpy(np.concatenate(parts))
    if torch.device(device).type == "cuda":
        host = host.pin_memory()
    dev = host.to(device, non_blocking=True)
    return list(dev.split(sizes))


def unsupported_reason(cfg) -> str | None:
    """Why a configuration must use the object path (``None`` when the device path applies).

    Vanilla and mixed blocks run on the device path's per-layer route with their dropout
    (attention probabilities, branch outputs, MLP activation) drawn from counter-based
    Philox streams; PRA blocks have no dropout (``src/pra_torch/model.py:31-167``)."""
    head_dim = cfg.d_model // cfg.n_heads
    checks = [
        (cfg.search_strategy not in ("hierarchical", "global_chunks"), f"search_strategy={cfg.search_strategy}"),
        (cfg.search_strategy == "global_chunks" and cfg.detail_materialization == "full_reference",
         "global_chunks with full-reference expansion"),
        (cfg.routing_backend != "tensorized", "legacy routing backend"),
        (cfg.use_summary, "summary routing"),
        (cfg.cache_build_mode != "detached", "trainable gists"),
        (cfg.reference_encoding_strategy != "independent", "grouped encoding"),
        (cfg.encoding_chunking is not None, "bounded encoding"),
        (cfg.gist_mode not in {"mean", "kmeans", "last", "ref_end"}, f"gist_mode={cfg.gist_mode}"),
        (cfg.gist_mode == "kmeans" and cfg.gist_kmeans_empty_cluster_policy == "error",
         "k-means error-on-empty-cluster policy"),
        (cfg.reference_level_gist_mode is not None, "URI-level gists"),
        (cfg.gists_per_chunk > 8, "more than 8 gists"),
        (head_dim not in (16, 32, 64, 128), f"head_dim={head_dim}"),
        (cfg.d_model % 8 or cfg.d_ff % 8, "widths not multiple of 8"),
        (cfg.collect_routing_metrics or cfg.collect_rank_diagnostics, "full ranking diagnostics"),
        (cfg.collect_detailed_timing, "host-timed diagnostics"),
    ]
    for bad, reason in checks:
        if bad:
            return reason
    return None


# ---------------------------------------------------------------------------
# Flat parameters
# ---------------------------------------------------------------------------

def _round(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def block_kind(block) -> str:
    """``"pra"`` (PRA block), ``"vanilla"`` (causal encoder block, no memory) or ``"mixed"``
    (vanilla self-attention residual, then a PRA residual, then the MLP)."""
    name = type(block).__name__
    if name == "VanillaTransformerBlock":
        return "vanilla"
    if name == "PRASATransformerBlock":
        return "mixed"
    return "pra"


class FlatParams:
    """fp32 master / bf16 compute / bf16 gradient / AdamW moment buffers in one layout."""

    def __init__(self, model: TinyPRAModel, vocab_pad: int):
        self.model = model
        ordered = self._ordered(model)
        offsets, cursor = {}, 0
        for name, p in ordered:
            offsets[name] = cursor
            cursor += _round(p.numel())
        head = model.head.weight
        self.head_offset = offsets["head.weight"]
        # the head's bf16 view is padded to vocab_pad rows of zeros (TMA-friendly logits width)
        self.total = cursor + _round((vocab_pad - head.shape[0]) * head.shape[1])
        dev = head.device
        self.master = torch.zeros(self.total, device=dev, dtype=torch.float32)
        self.shadow = torch.zeros(self.total, device=dev, dtype=torch.bfloat16)
        self.grad = torch.zeros(self.total, device=dev, dtype=torch.bfloat16)
        self.exp_avg = torch.zeros(self.total, device=dev, dtype=torch.float32)
        self.exp_avg_sq = torch.zeros(self.total, device=dev, dtype=torch.float32)
        self.offsets = offsets
        self.params = dict(ordered)
        for name, p in ordered:
            view = self.master[offsets[name]: offsets[name] + p.numel()].view_as(p)
            view.copy_(p.data)
            p.data = view
        self.vocab_pad = vocab_pad
        self.refresh_shadow()

    @staticmethod
    def _ordered(model: TinyPRAModel) -> list[tuple[str, torch.nn.Parameter]]:
        """Parameters in flat-buffer order: each block's parameters contiguous (q, k, v adjacent
        so one [3D, D] span serves the fused QKV GEMM), then embeddings, final norm, head."""
        named = dict(model.named_parameters())
        order = []
        for i, block in enumerate(model.blocks):
            pre = f"blocks.{i}."
            kind = block_kind(block)
            if kind == "vanilla":
                lay = pre + "layer."
                order += [lay + "self_attn.in_proj_weight", lay + "self_attn.in_proj_bias",
                          lay + "self_attn.out_proj.weight", lay + "self_attn.out_proj.bias", lay + "norm1.weight",
                          lay + "norm1.bias", lay + "norm2.weight", lay + "norm2.bias", lay + "linear1.weight",
                          lay + "linear1.bias", lay + "linear2.weight", lay + "linear2.bias"]
                continue
            attn = pre + ("pra_attn." if kind == "mixed" else "attn.")
            if kind == "mixed":
                order += [pre + "self_attn.in_proj_weight", pre + "self_attn.in_proj_bias",
                          pre + "self_attn.out_proj.weight", pre + "self_attn.out_proj.bias"]
            for proj in ("q_proj", "k_proj", "v_proj"):
                order.append(attn + f"{proj}.weight")
            for proj in ("q_proj", "k_proj", "v_proj"):
                order.append(attn + f"{proj}.bias")
            order += [attn + "o_proj.weight", attn + "o_proj.bias", pre + "ln1.weight", pre + "ln1.bias",
                      pre + "ln2.weight", pre + "ln2.bias"]
            if kind == "mixed":
                order += [pre + "ln3.weight", pre + "ln3.bias", pre + "ff.0.weight", pre + "ff.0.bias",
                          pre + "ff.3.weight", pre + "ff.3.bias"]
            else:
                order += [pre + "ff.0.weight", pre + "ff.0.bias", pre + "ff.2.weight", pre + "ff.2.bias"]
        order += ["token_emb.weight", "pos_emb.weight", "ln.weight", "ln.bias"]
        order += [n for n in named if n not in order and n != "head.weight"]
        order.append("head.weight")
        return [(n, named[n]) for n in order]

    def refresh_shadow(self) -> None:
        self.shadow.copy_(self.master)

    def rehome_grad(self, new: torch.Tensor, views: list[torch.Tensor]) -> None:
        """Move the gradient buffer into ``new`` (e.g. symmetric memory) without
        rebuilding anything: every view in ``views`` (slot gradients, embedding
        gradients) is re-pointed in place at the same offset of ``new``."""
        old = self.grad
        assert new.numel() == old.numel() and new.dtype == old.dtype and new.is_contiguous()
        new.copy_(old)
        base = old.storage_offset()
        storage = new.untyped_storage()
        for v in views:
            v.set_(storage, new.storage_offset() + v.storage_offset() - base, v.size(), v.stride())
        self.grad = new

    def view(self, buffer: torch.Tensor, name: str, rows: int | None = None) -> torch.Tensor:
        p = self.params[name]
        if rows is None:
            return buffer[self.offsets[name]: self.offsets[name] + p.numel()].view_as(p)
        return buffer[self.offsets[name]: self.offsets[name] + rows * p.shape[1]].view(rows, p.shape[1])

    def span(self, buffer: torch.Tensor, first: str, count: int, shape) -> torch.Tensor:
        """A contiguous view covering ``count`` elements starting at parameter ``first``."""
        start = self.offsets[first]
        return buffer[start: start + count].view(*shape)

    def slot(self, weight: str, bias: str | None = None) -> WeightSlot:
        return WeightSlot(w=self.view(self.shadow, weight), b=self.view(self.shadow, bias) if bias else None,
                          gw=self.view(self.grad, weight), gb=self.view(self.grad, bias) if bias else None)


class FusedAdamW(torch.optim.Optimizer):
    """AdamW over the flat buffers (one clip-norm reduction + one update kernel per step).

    Parameter groups expose ``lr`` / ``betas`` / ``eps`` / ``weight_decay`` so the
    stock ``LambdaLR`` warm-up and checkpoint round trips work unchanged.
    """

    def __init__(self, flat: FlatParams, lr: float, weight_decay: float, betas=(0.9, 0.999), eps: float = 1e-8,
                 max_grad_norm: float = 1.0):
        super().__init__(list(flat.params.values()), dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.flat = flat
        self.max_grad_norm = max_grad_norm
        self.step_count = 0
        self.last_norm = None
        self.grad_source = None  # set by the data-parallel engine to its reduced fp32 buffer
        self.grad_scale = 1.0    # 1/world when grad_source holds a sum over ranks

    def zero_grad(self, set_to_none: bool = True) -> None:
        for s in getattr(self.flat, "slots", ()):
            s.fresh[0] = True

    @torch.no_grad()
    @traced("pra.optimizer")
    def step(self, closure=None):
        ext = _ext.require()
        group = self.param_groups[0]
        grads = self.grad_source if self.grad_source is not None else self.flat.grad
        # clip on the averaged gradient: ||sum / world|| = ||sum|| / world
        norm, coef = ext.grad_norm(grads, float(self.max_grad_norm) / self.grad_scale)
        self.step_count += 1
        b1, b2 = group["betas"]
        ext.adamw(self.flat.master, self.flat.shadow, grads, self.flat.exp_avg, self.flat.exp_avg_sq,
                  float(group["lr"]), b1, b2, float(group["eps"]), float(group["weight_decay"]), self.step_count,
                  coef, float(self.grad_scale))
        if self.grad_scale != 1.0:
            norm = norm * self.grad_scale
        self.last_norm = norm
        return None

    def state_dict(self):
        base = super().state_dict()
        base["fused"] = {"step": self.step_count, "exp_avg": self.flat.exp_avg.cpu(),
                         "exp_avg_sq": self.flat.exp_avg_sq.cpu()}
        return base

    def load_state_dict(self, state_dict):
        fused = state_dict.get("fused")
        if fused is not None:
            self.step_count = int(fused["step"])
            self.flat.exp_avg.copy_(fused["exp_avg"])
            self.flat.exp_avg_sq.copy_(fused["exp_avg_sq"])
        for group, saved in zip(self.param_groups, state_dict["param_groups"]):
            for key in ("lr", "betas", "eps", "weight_decay", "initial_lr"):
                if key in saved:
                    group[key] = saved[key]


# ---------------------------------------------------------------------------
# Batched cache plan
# ---------------------------------------------------------------------------

@dataclass
class ChunkRecord:
    row: int
    entry: int           # global entry index
    uri: str
    chunk_id: str
    token_start: int
    token_end: int
    token_ids: tuple
    seq: int = -1        # encode sequence (pool rows seq * L .. seq * L + len)
    metadata: dict = field(default_factory=dict)


@dataclass
class EntryRecord:
    row: int
    uri: str
    text: str
    metadata: dict
    use_memory: bool
    visible: tuple        # global entry indices readable while this entry encodes
    chunks: list = field(default_factory=list)  # global chunk indices
    wave: int = 0


class Namespace:
    """Device arrays describing row-local routing namespaces (see ``RouteParams``)."""

    def __init__(self, rows_entries: list[list[int]], entries: list[EntryRecord], chunks: list[ChunkRecord],
                 device, arrays: list[torch.Tensor] | None = None):
        if arrays is None:
            host = self.host_arrays(rows_entries, entries, chunks)
            arrays = _upload(device, *host)
            empty = len(host[3]) == 0
        else:
            empty = bool(getattr(arrays, "empty", False))
        (self.row_pos_off, self.row_ref_off, self.ref_pos_off, self.pos_chunk, self.pos_ref,
         self.pos_rank) = arrays
        self.rows_entries = rows_entries
        self.empty = empty

    @staticmethod
    def host_arrays(rows_entries, entries, chunks) -> list[list[int]]:
        row_pos_off, row_ref_off, ref_pos_off = [0], [0], [0]
        pos_chunk, pos_ref, pos_rank = [], [], []
        for entry_ids in rows_entries:
            by_uri = sorted(entry_ids, key=lambda e: entries[e].uri)
            for local_ref, e in enumerate(by_uri):
                ids = entries[e].chunks
                rank = {c: i for i, c in enumerate(sorted(ids, key=lambda c: chunks[c].chunk_id))}
                for c in ids:
                    pos_chunk.append(c)
                    pos_ref.append(local_ref)
                    pos_rank.append(rank[c])
                ref_pos_off.append(len(pos_chunk))
            row_pos_off.append(len(pos_chunk))
            row_ref_off.append(len(ref_pos_off) - 1)
        return [row_pos_off, row_ref_off, ref_pos_off, pos_chunk, pos_ref, pos_rank]


class BatchMemory:
    """All rows' encoded references of one batch: pools, gists and chunk tables per layer."""

    def __init__(self, runtime, entries, chunks, rows, seq_len, device, chunk_tables=None, prompt_ns=None):
        cfg = runtime.cfg
        self.entries, self.chunks, self.rows = entries, chunks, rows
        self.seq_len = seq_len
        n_seq = max(len(chunks), 1)
        width = 3 * cfg.d_model
        L = cfg.n_layers
        # one allocation per table; per-layer views keep the indexing simple
        self.pool = torch.empty((L, n_seq * seq_len, width), device=device, dtype=torch.bfloat16)
        self.pools = list(self.pool.unbind(0))
        self.kv_bytes = 0         # cached K/V bytes (bf16 keys + values of every chunk token and layer)
        self.device_kv_bytes = 0  # of which on the device (0 once the pool moves to the host tier)
        g = max(cfg.gists_per_chunk if cfg.gist_mode == "kmeans" else 1, 1)
        self.G = g
        self.n_seq = n_seq
        self.gist_tables = torch.zeros((3, L, n_seq, g, cfg.d_model), device=device, dtype=torch.float32)
        self.gists_all, self.gist_k_all, self.gist_v_all = self.gist_tables.unbind(0)
        self.gists = list(self.gists_all.unbind(0))
        self.gist_k = list(self.gist_k_all.unbind(0))
        self.gist_v = list(self.gist_v_all.unbind(0))
        self.gist_count_all = torch.zeros((L, n_seq), device=device, dtype=torch.int32)
        self.gist_count = list(self.gist_count_all.unbind(0))
        if chunk_tables is None:
            chunk_tables = _upload(device, [c.token_start for c in chunks], [len(c.token_ids) for c in chunks],
                                   [c.seq * seq_len for c in chunks])
        self.chunk_start, self.chunk_len, self.chunk_pool_row = chunk_tables
        self.prompt_ns = prompt_ns  # (device arrays, empty) of the prompt's namespace, when planned natively

    def k_view(self, layer: int, d: int) -> torch.Tensor:
        return self.pools[layer][:, d:2 * d]

    def v_view(self, layer: int, d: int) -> torch.Tensor:
        return self.pools[layer][:, 2 * d:]

    def k_all(self, d: int) -> torch.Tensor:
        """[L, rows, d] view of every layer's keys."""
        return self.pool[:, :, d:2 * d]

    def v_all(self, d: int) -> torch.Tensor:
        return self.pool[:, :, 2 * d:]


@dataclass
class LayerRouting:
    """Device outputs of one routing call (kept for deferred traces / metrics)."""

    mem_idx: torch.Tensor
    ints: torch.Tensor
    sel_i: torch.Tensor
    sel_f: torch.Tensor


@dataclass
class RowPlan:
    """Host-side plan of one row (row-local entry / chunk numbering)."""

    item: dict
    cache: object
    builder: object
    entries: list
    chunks: list


@dataclass
class BatchPlan:
    """Host-side cache-build plan of one batch (see ``DeviceRuntime.plan_batch``)."""

    metadata_rows: list
    caches: list
    builders: list
    entries: list
    chunks: list
    rows: list
    seq_len: int
    waves: list
    wave_tables: list | None = None   # per wave: {name: (offset, count)} into ``packed``
    packed: object | None = None      # every wave's int32 host tables in one array (one upload)


class KMeansTables:
    """Device copies of the seeded k-means initialisation draws, one block per chunk length.

    The seeded CPU generator's draws depend only on (chunk length, gist count,
    seed), so each distinct length is drawn once, appended to a device buffer and
    shared by every chunk of that length; a wave then ships only two offsets per
    chunk.  ``kmeans++`` blocks hold the first index and ``count - 1`` rows of
    Exp(1) draws; ``sample`` blocks hold the sampled point indices.
    """

    def __init__(self, cfg, device):
        self.cfg, self.device = cfg, device
        self.blocks: dict[int, tuple[int, int]] = {}
        self._draws: list[torch.Tensor] = []
        self._idx: list[int] = []
        self._draw_cursor = 0
        self.draws = torch.zeros(1, device=device)
        self.idx = torch.zeros(1, dtype=torch.int32, device=device)

    def lookup(self, lengths: list[int]) -> tuple[list[int], list[int]]:
        cfg = self.cfg
        new = [n for n in dict.fromkeys(lengths) if n not in self.blocks]
        for n in new:
            count = min(max(cfg.gists_per_chunk, 1), n)
            if cfg.gist_kmeans_init == "kmeans++":
                first, exp = kmeanspp_random_stream(n, count, cfg.gist_kmeans_seed)
                self.blocks[n] = (int(first), self._draw_cursor)
                self._draws.append(exp.flatten().float())
                self._draw_cursor += exp.numel()
            else:
                perm = torch.randperm(n, generator=local_generator(cfg.gist_kmeans_seed))[:count]
                self.blocks[n] = (len(self._idx), 0)
                self._idx.extend(int(i) for i in perm)
        if new:  # rare: a chunk length not seen before
            if self._draws:
                self.draws = torch.cat(self._draws).to(self.device)
            if self._idx:
                self.idx = torch.tensor(self._idx, dtype=torch.int32).to(self.device)
        firsts = [self.blocks[n][0] for n in lengths]
        offs = [self.blocks[n][1] for n in lengths]
        return firsts, offs


# ---------------------------------------------------------------------------
# Runtime
# ---------------------------------------------------------------------------

class DeviceRuntime:
    def __init__(self, model: TinyPRAModel):
        self.model = model
        self.cfg = model.cfg
        cfg = self.cfg
        self.device = model.head.weight.device
        self.head_dim = cfg.d_model // cfg.n_heads
        self.vocab_pad = (cfg.vocab_size + 127) // 128 * 128
        self.flat = FlatParams(model, self.vocab_pad)
        f = self.flat
        d = cfg.d_model
        self.layers = []
        self.kinds = [block_kind(block) for block in model.blocks]
        for i, kind in enumerate(self.kinds):
            pre = f"blocks.{i}."
            if kind == "vanilla":
                lay = pre + "layer."
                self.layers.append({
                    "ln1": f.slot(lay + "norm1.weight", lay + "norm1.bias"),
                    "qkv": f.slot(lay + "self_attn.in_proj_weight", lay + "self_attn.in_proj_bias"),
                    "o": f.slot(lay + "self_attn.out_proj.weight", lay + "self_attn.out_proj.bias"),
                    "ln2": f.slot(lay + "norm2.weight", lay + "norm2.bias"),
                    "up": f.slot(lay + "linear1.weight", lay + "linear1.bias"),
                    "down": f.slot(lay + "linear2.weight", lay + "linear2.bias"),
                })
                continue
            attn = pre + ("pra_attn." if kind == "mixed" else "attn.")
            qkv = WeightSlot(w=f.span(f.shadow, attn + "q_proj.weight", 3 * d * d, (3 * d, d)),
                             b=f.span(f.shadow, attn + "q_proj.bias", 3 * d, (3 * d,)),
                             gw=f.span(f.grad, attn + "q_proj.weight", 3 * d * d, (3 * d, d)),
                             gb=f.span(f.grad, attn + "q_proj.bias", 3 * d, (3 * d,)))
            self._check_contiguous(attn)
            if kind == "mixed":  # the PRA branch's norms are ln2 (attention) and ln3 (MLP)
                self.layers.append({
                    "ln1": f.slot(pre + "ln2.weight", pre + "ln2.bias"), "qkv": qkv,
                    "o": f.slot(attn + "o_proj.weight", attn + "o_proj.bias"),
                    "ln2": f.slot(pre + "ln3.weight", pre + "ln3.bias"),
                    "up": f.slot(pre + "ff.0.weight", pre + "ff.0.bias"),
                    "down": f.slot(pre + "ff.3.weight", pre + "ff.3.bias"),
                    "sa_ln": f.slot(pre + "ln1.weight", pre + "ln1.bias"),
                    "sa_qkv": f.slot(pre + "self_attn.in_proj_weight", pre + "self_attn.in_proj_bias"),
                    "sa_o": f.slot(pre + "self_attn.out_proj.weight", pre + "self_attn.out_proj.bias"),
                })
                continue
            self.layers.append({
                "ln1": f.slot(pre + "ln1.weight", pre + "ln1.bias"), "qkv": qkv,
                "o": f.slot(attn + "o_proj.weight", attn + "o_proj.bias"),
                "ln2": f.slot(pre + "ln2.weight", pre + "ln2.bias"),
                "up": f.slot(pre + "ff.0.weight", pre + "ff.0.bias"),
                "down": f.slot(pre + "ff.2.weight", pre + "ff.2.bias"),
            })
        self.cross_attention = cfg.memory_transport == "cross_attention"
        if self.cross_attention:  # legacy transport: the memory branch has its own output projection
            for i, (kind, layer) in enumerate(zip(self.kinds, self.layers)):
                if kind != "vanilla":
                    attn = f"blocks.{i}." + ("pra_attn." if kind == "mixed" else "attn.")
                    layer["mem_o"] = f.slot(attn + "mem_o_proj.weight", attn + "mem_o_proj.bias")
        # vanilla / mixed blocks and the cross-attention transport run the per-layer path (the
        # native stacks hold native-K/V PRA blocks only)
        self.uniform_pra = all(kind == "pra" for kind in self.kinds) and not self.cross_attention
        self.dropout_streams = DropoutStreams()
        self._host_pool: torch.Tensor | None = None  # pinned K/V pool of the CPU-resident tier
        self._retired_host_pools: list[torch.Tensor] = []
        self.ln_f = f.slot("ln.weight", "ln.bias")
        head_rows = self.vocab_pad
        self.head = WeightSlot(w=f.view(f.shadow, "head.weight", rows=head_rows),
                               gw=f.view(f.grad, "head.weight", rows=head_rows))
        f.slots = [s for layer in self.layers for s in layer.values()] + [self.ln_f, self.head]
        self.tok_emb_w = f.view(f.shadow, "token_emb.weight")
        self.pos_emb_w = f.view(f.shadow, "pos_emb.weight")
        self.tok_emb_g = f.view(f.grad, "token_emb.weight")
        self.pos_emb_g = f.view(f.grad, "pos_emb.weight")
        self.anchor = torch.zeros(1, device=self.device, requires_grad=True)  # puts embeddings on the tape
        self.kmeans_tables = KMeansTables(cfg, self.device)
        self._prefetched_rows: tuple | None = None  # (metadata rows, {row: RowPlan})
        self._prefetched_native: tuple | None = None  # (metadata rows, NativeBatchPlan)
        self.upcoming: list | None = None  # next batch's rows, planned in slices during this step
        self._last_tokenizer = None
        self._last_resolver = None
        self.last_routing: dict[int, LayerRouting] = {}
        self.last_memory: BatchMemory | None = None
        self.last_namespace: Namespace | None = None

    @classmethod
    def for_planning(cls, model: TinyPRAModel, device="cpu") -> "DeviceRuntime":
        """A runtime that only plans cache builds (no parameters, no device buffers): the
        host half of the device path, usable without a GPU."""
        rt = cls.__new__(cls)
        rt.model, rt.cfg, rt.device = model, model.cfg, torch.device(device)
        rt.kmeans_tables = KMeansTables(model.cfg, rt.device)
        rt._prefetched_rows = rt._prefetched_native = None
        rt.upcoming = rt._last_tokenizer = rt._last_resolver = None
        return rt

    grad_hooks = None  # optional: before_stack() / after_layer(l) calls during the backward
    route_timer = None  # optional list: (start, end) CUDA events around each per-layer routing launch

    def grad_views(self) -> list[torch.Tensor]:
        """Every tensor that aliases the flat gradient buffer."""
        views = [t for slot in self.flat.slots for t in (slot.gw, slot.gb) if t is not None]
        return views + [self.tok_emb_g, self.pos_emb_g]

    def _check_contiguous(self, attn: str) -> None:
        f = self.flat
        d = self.cfg.d_model
        if (f.offsets[attn + "k_proj.weight"] != f.offsets[attn + "q_proj.weight"] + d * d
                or f.offsets[attn + "v_proj.bias"] != f.offsets[attn + "q_proj.bias"] + 2 * d):
            raise RuntimeError("q/k/v parameters must be adjacent in the flat layout (d_model*d_model % 64 != 0?)")

    # -- embeddings -----------------------------------------------------------
    def embed(self, ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        return _Embed.apply(ids, positions, self.anchor, self)

    # -- one decoder pass ---------------------------------------------------------
    def run_blocks(self, x: torch.Tensor, b: int, t: int, key_valid, routing, memory: BatchMemory | None,
                   stop_after_kv: bool = False, pool_rows: slice | None = None, budget: int = 0,
                   query_rows: torch.Tensor | None = None, after_qkv=None):
        """Run the block stack on ``x`` ``[b*t, D]``.

        ``routing`` is a ``Namespace`` (or ``None`` for no memory); with ``pool_rows``
        the QKV of every layer is written into those rows of the layer pool (cache
        build).  ``stop_after_kv`` skips the last block's attention and MLP.
        ``after_qkv(layer)`` runs after each layer's QKV projection (no-grad native
        stack only): the layer-synchronous cache build computes that layer's gists there.
        """
        cfg = self.cfg
        d = cfg.d_model
        if query_rows is not None:
            query_rows = query_rows.to(torch.int32)
        if not self.uniform_pra:
            return self._run_blocks_layerwise(x, b, t, key_valid, routing, memory, stop_after_kv, pool_rows, budget,
                                              query_rows, after_qkv)
        if not torch.is_grad_enabled():
            return self._run_blocks_native(x, b, t, key_valid, routing, memory, stop_after_kv, pool_rows, budget,
                                           query_rows, after_qkv)
        if after_qkv is not None:
            raise RuntimeError("per-layer hooks run only in the no-grad native stack")
        if pool_rows is None and not stop_after_kv and _NATIVE_TRAIN_STACK:
            return _TrainStack.apply(x, self, b, t, key_valid, routing, memory, budget, query_rows)
        return self._run_blocks_layerwise(x, b, t, key_valid, routing, memory, stop_after_kv, pool_rows, budget,
                                          query_rows, None)

    def _dropout(self) -> float:
        """Dropout probability of the vanilla / mixed blocks now (training mode only; PRA blocks
        have none, ``src/pra_torch/model.py:31-167``)."""
        return float(self.cfg.dropout) if self.model.training and not self.uniform_pra else 0.0

    def _self_attention(self, x, layer, prefix: str, b: int, t: int, key_valid, p: float, residual_dropout: bool):
        """``x + [dropout](out_proj(causal MHA(norm(x))))`` of a vanilla block (``prefix`` "") or of
        a mixed block's leading sublayer (``prefix`` "sa_"; no dropout on its output)."""
        cfg = self.cfg
        d = cfg.d_model
        h = layer_norm(x, layer[prefix + "ln1" if not prefix else "sa_ln"])
        qkv = linear(h, layer[prefix + "qkv"])
        streams = self.dropout_streams
        a = attention(qkv.view(b, t, 3 * d), cfg.n_heads, self.head_dim, None, key_valid, drop=streams.next(p))
        if residual_dropout and p > 0.0:
            return dropout_add(x, linear(a.view(b * t, d), layer[prefix + "o"]), streams.next(p))
        return linear(a.view(b * t, d), layer[prefix + "o"], residual=x)

    def _cross_attention(self, x, qkv3, layer, mem: MemoryView | None, key_valid, b: int, t: int):
        """Legacy ``cross_attention`` transport (``src/pra_torch/attention.py:557-628``): local causal
        attention through ``o_proj`` plus ``memory_alpha`` times a separately normalised attention
        over the row's selected memory keys through ``mem_o_proj``; rows without memory add
        nothing.  The memory branch is the ragged kernel with every local key masked."""
        cfg = self.cfg
        d = cfg.d_model
        a = attention(qkv3, cfg.n_heads, self.head_dim, None, key_valid)
        x = linear(a.view(b * t, d), layer["o"], residual=x)
        if mem is None:
            return x
        hidden = torch.zeros((b, t), device=qkv3.device, dtype=torch.uint8)  # no local key is visible
        am = attention(qkv3, cfg.n_heads, self.head_dim, mem, hidden)
        m = linear(am.view(b * t, d), layer["mem_o"])
        rows = (mem.length > 0).to(m.dtype) * float(cfg.memory_alpha)
        return x + m * rows.repeat_interleave(t)[:, None]

    def _run_blocks_layerwise(self, x, b, t, key_valid, routing, memory, stop_after_kv, pool_rows, budget,
                              query_rows, after_qkv):
        """Per-layer path (autograd ops over the same kernels): every block kind, dropout in the
        vanilla and mixed blocks, and the cache build's pool writes and gist hook."""
        cfg = self.cfg
        d = cfg.d_model
        p = self._dropout()
        streams = self.dropout_streams
        last = len(self.layers) - 1
        for li, (kind, layer) in enumerate(zip(self.kinds, self.layers)):
            if kind == "vanilla":
                if pool_rows is not None:  # nothing routes at a vanilla layer; keep its pool rows defined
                    memory.pools[li][pool_rows].zero_()
                if stop_after_kv and li == last:
                    return None
                x = self._self_attention(x, layer, "", b, t, key_valid, p, residual_dropout=True)
                x = mlp(layer_norm(x, layer["ln2"]), x, layer["up"], layer["down"], streams.next(p), streams.next(p))
                continue
            if kind == "mixed":
                x = self._self_attention(x, layer, "sa_", b, t, key_valid, p, residual_dropout=False)
            h = layer_norm(x, layer["ln1"])
            if pool_rows is not None:
                qkv = memory.pools[li][pool_rows]
                _ext.require().gemm("tn", h, layer["qkv"].w, None, qkv, layer["qkv"].b, None, 1.0, 0.0, None)
            else:
                qkv = linear(h, layer["qkv"])
            if after_qkv is not None:
                after_qkv(li)
            if stop_after_kv and li == last:
                return None
            qkv3 = qkv.view(b, t, 3 * d)
            mem = None
            if routing is not None and not routing.empty:
                mem = self.route(li, qkv3, routing, memory, budget, query_rows)
            if self.cross_attention:
                x = self._cross_attention(x, qkv3, layer, mem, key_valid, b, t)
            else:
                a = attention(qkv3, cfg.n_heads, self.head_dim, mem, key_valid)
                x = linear(a.view(b * t, d), layer["o"], residual=x)
            drop_in = streams.next(p) if kind == "mixed" else None  # the mixed MLP's dropout after GELU
            x = mlp(layer_norm(x, layer["ln2"]), x, layer["up"], layer["down"], drop_in)
        return x

    def _route_settings(self, budget) -> tuple[list[float], torch.Tensor | None]:
        """(route_cfg list of the native executor / route binding, per-row budget tensor or None)."""
        cfg = self.cfg
        max_sel = max(1, min(256, cfg.top_k_references * cfg.top_k_chunks_per_reference
                             if cfg.detail_materialization != "full_reference" else 256))
        budget_rows = budget if torch.is_tensor(budget) else None
        scalar_budget = int(budget) if budget_rows is None else cfg.effective_model_max_context_tokens
        settings = [min(cfg.top_k_references, 64), cfg.top_k_chunks_per_reference, _AGG[cfg.gist_score_aggregation],
                    _AGG[cfg.reference_score_aggregation], float(cfg.trigger_threshold), scalar_budget,
                    float(cfg.detail_materialization == "gist_only"),
                    float(cfg.detail_materialization == "full_reference"),
                    float(cfg.overlap_materialization == "deduplicate"), max_sel, max(scalar_budget, 1),
                    float(cfg.search_strategy == "global_chunks")]
        return settings, budget_rows

    def _stack_weights(self) -> list[torch.Tensor]:
        if getattr(self, "_stack_weight_list", None) is None:
            out = []
            for layer in self.layers:
                for name in ("ln1", "qkv", "o", "ln2", "up", "down"):
                    out += [layer[name].w, layer[name].b]
            self._stack_weight_list = out
        return self._stack_weight_list

    def _run_blocks_native(self, x, b, t, key_valid, routing, memory, stop_after_kv, pool_rows, budget, query_rows,
                           after_qkv=None):
        """The whole block stack in one native call (no autograd): cache build and no-grad forwards."""
        cfg = self.cfg
        d = cfg.d_model
        ext = _ext.require()
        routed = routing is not None and not routing.empty
        ns, gists, counts, gist_kv, budget_rows, settings = [], None, None, None, None, []
        if routed:
            ns = [routing.row_pos_off, routing.row_ref_off, routing.ref_pos_off, routing.pos_chunk, routing.pos_ref,
                  routing.pos_rank, memory.chunk_start, memory.chunk_len, memory.chunk_pool_row]
            gists, counts = memory.gists_all, memory.gist_count_all
            settings, budget_rows = self._route_settings(budget)
            if cfg.detail_materialization == "gist_only":
                gist_kv = torch.stack([memory.gist_k_all, memory.gist_v_all]).view(
                    2, cfg.n_layers, -1, d).bfloat16()
        pool = memory.pool if pool_rows is not None else None
        row0 = pool_rows.start if pool_rows is not None else 0
        out = ext.stack_forward(x.contiguous(), b, t, self._stack_weights(), cfg.n_heads, self.head_dim, 1e-5,
                                key_valid, pool, row0, stop_after_kv, memory.pool if routed else None, ns, gists,
                                counts, gist_kv, budget_rows,
                                query_rows, settings, after_qkv)
        n_layers = cfg.n_layers
        per_layer = 7 + (1 if routed else 0)
        _ext.add_launches("stack_forward", n_layers * per_layer - (per_layer - 2 if stop_after_kv else 0))
        # (gist launches made by after_qkv go through the counted extension proxy)
        if routed:
            for li in range(n_layers - (1 if stop_after_kv else 0)):
                mem_idx, ints, sel_i, sel_f = out[1 + 4 * li: 5 + 4 * li]
                self.last_routing[li] = LayerRouting(mem_idx, ints, sel_i, sel_f)
        return None if stop_after_kv else out[0]

    def route(self, li: int, qkv3: torch.Tensor, ns: Namespace, memory: BatchMemory, budget,
              query_rows: torch.Tensor | None) -> MemoryView:
        cfg = self.cfg
        d = cfg.d_model
        settings, budget_rows = self._route_settings(budget)
        gist_only = bool(settings[6])
        if query_rows is None:
            query_rows = torch.full((qkv3.shape[0],), qkv3.shape[1] - 1, dtype=torch.int32, device=qkv3.device)
        timer = self.route_timer
        if timer is not None:  # device time of each routing launch (systems benchmarks)
            timer.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
            timer[-1][0].record()
        mem_idx, ints, sel_i, sel_f = _ext.require().route(
            qkv3[:, :, :d], memory.gists[li], memory.gist_count[li], ns.row_pos_off, ns.row_ref_off, ns.ref_pos_off,
            ns.pos_chunk, ns.pos_ref, ns.pos_rank, memory.chunk_start, memory.chunk_len, memory.chunk_pool_row,
            int(settings[0]), int(settings[1]), int(settings[2]), int(settings[3]), settings[4], int(settings[5]),
            gist_only, bool(settings[7]), bool(settings[8]), int(settings[9]), int(settings[10]), budget_rows,
            query_rows, bool(settings[11]))
        if timer is not None:
            timer[-1][1].record()
        self.last_routing[li] = LayerRouting(mem_idx, ints, sel_i, sel_f)
        if gist_only:
            gk = memory.gist_k[li].view(-1, d).bfloat16()
            gv = memory.gist_v[li].view(-1, d).bfloat16()
            return MemoryView(gk, gv, mem_idx, ints[0])
        return MemoryView(memory.k_view(li, d), memory.v_view(li, d), mem_idx, ints[0])

    # -- cache build ------------------------------------------------------------
    def plan_row(self, item: dict, tokenizer, resolver_config=None) -> "RowPlan":
        """Host planning of one row: trace its recursive build, tokenise and chunk each entry once.

        Entry and chunk indices in the result are row-local; ``plan_batch`` renumbers them.
        """
        cfg = self.cfg
        (cache,), (builder,) = plan_cache_builds(self.model, tokenizer, [item], resolver_config=resolver_config)
        # chunk texts are not kept here (only token ids and positions), and fixed windows use the
        # tokenizer only to decode those texts: skip the decode
        chunk_tok = _IdsOnlyTokenizer(tokenizer) if cfg.chunking_mode == "fixed" else tokenizer
        entries: list[EntryRecord] = []
        chunks: list[ChunkRecord] = []
        limit = cfg.effective_model_max_context_tokens
        index_of = {}
        for step in builder.plan:
            ids = list(step.token_ids) if step.token_ids is not None else list(tokenizer.encode(step.text))
            if len(ids) > limit:
                raise _Unsupported("reference longer than the native limit needs bounded encoding")
            e = len(entries)
            index_of[step.uri] = e
            record = EntryRecord(0, step.uri, step.text, step.metadata, step.use_pra_memory,
                                 tuple(index_of[u] for u in step.visible_uris if u in index_of))
            for chunk in partition_reference_tokens(step.uri, ids, chunk_tok, cfg, step.metadata,
                                                    text=step.text, max_chunk_tokens=limit):
                ids_c = tuple(chunk.token_ids[:limit])
                record.chunks.append(len(chunks))
                chunks.append(ChunkRecord(0, e, step.uri, chunk.chunk_id, chunk.token_start,
                                          min(chunk.token_start + len(ids_c), chunk.token_end), ids_c,
                                          metadata=dict(chunk.metadata)))
            record.wave = (1 + max((entries[v].wave for v in record.visible), default=-1)) if record.use_memory \
                else 0
            entries.append(record)
        return RowPlan(item, cache, builder, entries, chunks)

    def _single_pass(self) -> bool:
        """Whether the cache build runs as one layer-synchronous pass over every chunk.

        A chunk's layer-l attention reads only layer-l keys, values and gists of the
        entries it may see, and those depend only on layer l-1 states, so computing
        each layer for every chunk at once gives the values of an entry-by-entry
        build (what the dependency waves order).  Gist-only materialisation reads
        the gists as attention keys and keeps the wave order.
        """
        return _LAYER_SYNC and self.cfg.detail_materialization != "gist_only"

    def plan_native(self, metadata_rows: list[dict], tokenizer, resolver_config=None) -> NativeBatchPlan | None:
        """The batch plan from the native planner, or ``None`` when it needs the Python planner."""
        ext = _ext.load()
        if ext is None or not hasattr(ext, "plan_batch"):
            return None
        settings = native_config(self.cfg, ResolverServiceConfig.from_value(resolver_config))
        if settings is None:
            return None
        settings["single_pass"] = self._single_pass()
        rows = list(metadata_rows)
        out = ext.plan_batch(rows, tokenizer, settings)
        if out is None:
            return None
        plan = NativeBatchPlan(out, rows, lambda r: self.plan_row(rows[r], tokenizer, resolver_config))
        if self.cfg.gist_mode == "kmeans":
            plan.fill_kmeans(self.kmeans_tables)
        return plan

    def plan_batch(self, metadata_rows: list[dict], tokenizer, resolver_config=None,
                   row_plans: dict | None = None) -> "BatchPlan":
        """Host half of the cache build: every row's plan (taken from ``row_plans`` when
        prefetched), renumbered into one batch and ordered into dependency waves."""
        row_plans = row_plans or {}
        caches, builders = [], []
        entries: list[EntryRecord] = []
        chunks: list[ChunkRecord] = []
        rows: list[list[int]] = []
        for row, item in enumerate(metadata_rows):
            plan = row_plans.get(row)
            if plan is None or plan.item is not item:
                plan = self.plan_row(item, tokenizer, resolver_config)
            e0, c0 = len(entries), len(chunks)
            for record in plan.entries:
                record.row = row
                record.visible = tuple(v + e0 for v in record.visible)
                record.chunks = [c + c0 for c in record.chunks]
            for chunk in plan.chunks:
                chunk.row = row
                chunk.entry += e0
            entries.extend(plan.entries)
            chunks.extend(plan.chunks)
            rows.append(list(range(e0, len(entries))))
            caches.append(plan.cache)
            builders.append(plan.builder)
        seq_len = max((len(c.token_ids) for c in chunks), default=1)
        n_waves = max((e.wave for e in entries), default=-1) + 1
        seq = 0
        waves: list[list[int]] = []
        for wave in range(n_waves):
            members = []
            for e in entries:
                if e.wave == wave:
                    for c in e.chunks:
                        chunks[c].seq = seq
                        members.append(c)
                        seq += 1
            waves.append(members)
        if self._single_pass() and len(waves) > 1:  # one encode group, in encode-sequence order
            waves = [[c for members in waves for c in members]]
        plan = BatchPlan(metadata_rows, caches, builders, entries, chunks, rows, seq_len, waves)
        self._wave_tables(plan)
        return plan

    def _wave_tables(self, plan: "BatchPlan") -> None:
        """Every wave's host-side inputs (token ids, padding masks, budgets, routing
        namespaces, gist inputs) packed into one int32 array, so the cache build ships them
        to the device in a single pinned copy."""
        import numpy as np

        cfg = self.cfg
        L = plan.seq_len
        chunks, entries = plan.chunks, plan.entries
        limit = cfg.effective_model_max_context_tokens - cfg.context_safety_reserve_tokens
        cap = cfg.max_materialized_memory_tokens
        parts, tables, cursor = [], [], 0

        def put(table, name, values, dtype=np.int32):
            nonlocal cursor
            arr = np.asarray(values, dtype=dtype).ravel()
            if dtype == np.uint8:  # bytes ride in int32 words
                pad = (-arr.size) % 4
                words = np.concatenate([arr, np.zeros(pad, np.uint8)]).view(np.int32)
                table[name] = (cursor, int(words.size), int(arr.size))
                parts.append(words)
                cursor += words.size
                return
            if arr.size == 0:
                arr = np.zeros(1, np.int32)
            table[name] = (cursor, int(arr.size), int(arr.size))
            parts.append(arr)
            cursor += arr.size

        for members in plan.waves:
            t = {}
            n = len(members)
            lens = [len(chunks[c].token_ids) for c in members]
            ids = np.zeros((n, L), dtype=np.int32)
            for i, c in enumerate(members):
                ids[i, : lens[i]] = chunks[c].token_ids
            valid = (np.arange(L)[None, :] < np.asarray(lens)[:, None]).astype(np.uint8)
            put(t, "ids", ids)
            put(t, "valid", valid, np.uint8)
            put(t, "lens", lens)
            put(t, "last", [k - 1 for k in lens])
            put(t, "budget", [max(0, min(limit - k, cap) if cap is not None else limit - k) for k in lens])
            put(t, "gist_rows", [chunks[c].seq * L for c in members])
            put(t, "dest", members)
            if cfg.gist_mode == "kmeans":
                firsts, offs = self.kmeans_tables.lookup(lens)
                put(t, "km_first", firsts)
                put(t, "km_off", offs)
            rows_entries = None
            if any(entries[chunks[c].entry].use_memory for c in members):
                rows_entries = [list(entries[chunks[c].entry].visible) if entries[chunks[c].entry].use_memory else []
                                for c in members]
                host = Namespace.host_arrays(rows_entries, entries, chunks)
                for name, arr in zip(("ns0", "ns1", "ns2", "ns3", "ns4", "ns5"), host):
                    put(t, name, arr)
                t["ns_empty"] = len(host[3]) == 0
            t["rows_entries"] = rows_entries
            t["has_ns"] = rows_entries is not None
            t["n"], t["max_len"] = n, max(lens) if lens else 1
            tables.append(t)
        plan.wave_tables = tables
        plan.packed = np.concatenate(parts) if parts else np.zeros(1, np.int32)

    def prefetch(self, metadata_rows: list[dict], tokenizer=None, resolver_config=None, part: int = 0,
                 parts: int = 1) -> None:
        """Plan rows of the NEXT batch on the host while the device runs the current one.

        Planning needs no model state (only the tokenizer, resolver settings and the
        rows' reference tables), so doing it ahead is exact.  ``part``/``parts``
        plan a slice of the rows, so the work can be spread over several points of
        the current step; ``build_memory`` picks the plans up (and plans whatever is
        missing) when it is called with the same rows.
        """
        tokenizer = tokenizer or self._last_tokenizer
        if tokenizer is None:
            return
        resolver_config = resolver_config if resolver_config is not None else self._last_resolver
        if _NATIVE_PLANNER:
            if self._prefetched_native is not None and self._prefetched_native[0] is metadata_rows:
                return
            plan = self.plan_native(metadata_rows, tokenizer, resolver_config)
            if plan is not None:
                self._prefetched_native = (metadata_rows, plan)
                return
        if self._prefetched_rows is None or self._prefetched_rows[0] is not metadata_rows:
            self._prefetched_rows = (metadata_rows, {})
        done = self._prefetched_rows[1]
        n = len(metadata_rows)
        for row in range(part * n // parts, (part + 1) * n // parts):
            if row not in done:
                try:
                    done[row] = self.plan_row(metadata_rows[row], tokenizer, resolver_config)
                except _Unsupported:
                    return

    @traced("pra.cache_build")
    def build_memory(self, metadata_rows: list[dict], tokenizer, resolver_config=None):
        """Plan (or take the prefetched plan of) the batch, then encode all rows' chunks wave by wave."""
        self._last_tokenizer, self._last_resolver = tokenizer, resolver_config
        plan = None
        if self._prefetched_native is not None and self._prefetched_native[0] is metadata_rows:
            plan = self._prefetched_native[1]
        self._prefetched_native = None
        ready = {}
        if self._prefetched_rows is not None and self._prefetched_rows[0] is metadata_rows:
            ready = self._prefetched_rows[1]
        self._prefetched_rows = None
        if plan is None and _NATIVE_PLANNER and not ready:
            plan = self.plan_native(metadata_rows, tokenizer, resolver_config)
        if plan is None:
            plan = self.plan_batch(metadata_rows, tokenizer, resolver_config, ready)
            for cache, builder in zip(plan.caches, plan.builders):
                cache.resolution_events = list(builder.events)
                cache.dependencies = list(builder.dependencies)
        caches, builders, entries, chunks, rows, seq_len = (plan.caches, plan.builders, plan.entries, plan.chunks,
                                                            plan.rows, plan.seq_len)
        host = torch.from_numpy(plan.packed)
        if self.device.type == "cuda":
            host = host.pin_memory()
        packed = host.to(self.device, non_blocking=True)
        chunk_tables = prompt_ns = None
        if getattr(plan, "native", False):
            pt = plan.prompt_table
            view = lambda name: packed[pt[name][0]: pt[name][0] + pt[name][1]]  # noqa: E731
            chunk_tables = (view("chunk_start"), view("chunk_len"), view("chunk_pool_row"))
            prompt_ns = ([view(f"ns{i}") for i in range(6)], bool(pt["ns_empty"]))
        memory = BatchMemory(self, entries, chunks, rows, seq_len, self.device, chunk_tables, prompt_ns)
        if self.cfg.gist_mode in ("last", "ref_end"):
            self._single_gist_rows(plan, tokenizer)
        out = getattr(plan, "out", None)
        tokens = int(out["chunk_token_off"][-1]) if out is not None and len(out["chunk_token_off"]) else \
            sum(len(c.token_ids) for c in chunks)
        memory.kv_bytes = memory.device_kv_bytes = tokens * self.cfg.n_layers * 2 * self.cfg.d_model * 2
        with torch.no_grad():
            start = 0
            for wave_chunks, table in zip(plan.waves, plan.wave_tables):
                if not wave_chunks:
                    continue
                self._encode_wave(memory, wave_chunks, start, table, packed)
                start += len(wave_chunks)
        if self.cfg.kv_cache_residency == "cpu":
            self._move_pool_to_host(memory)
        self.last_memory = memory
        return memory, caches, builders

    def _single_gist_rows(self, plan, tokenizer) -> None:
        """``last`` / ``ref_end`` gists (``src/pra_torch/gists/single.py``): a chunk's gist is the
        key (and value) of one of its tokens -- the last one, or the reference terminator, which
        must occur exactly once in the chunk.  Each wave gets the pool row of that token and a
        length of one, so the mean-gist kernel reads exactly that row."""
        cfg = self.cfg
        marker = None
        if cfg.gist_mode == "ref_end":
            ids = list(tokenizer.encode(cfg.ref_end_token))
            if len(ids) != 1:
                raise ValueError(f"Reference terminator {cfg.ref_end_token!r} is not one atomic token.")
            marker = ids[0]
        packed, L = plan.packed, plan.seq_len
        for table in plan.wave_tables:
            if not table.get("n", table["lens"][2]):
                continue

            def host(name):
                off, _, count = table[name]
                return np.asarray(packed[off: off + count], dtype=np.int64)

            rows, lens = host("gist_rows"), host("lens")
            if marker is None:
                pick = np.maximum(lens - 1, 0)
            else:
                off = table["ids"][0]
                ids = np.asarray(packed[off: off + lens.size * L]).reshape(lens.size, L)
                hit = (ids == marker) & (np.arange(L)[None, :] < lens[:, None])
                counts = hit.sum(axis=1)
                if (counts[lens > 0] != 1).any():
                    bad = int(counts[lens > 0][counts[lens > 0] != 1][0])
                    raise ValueError(f"Expected exactly one {cfg.ref_end_token!r} token, found {bad}.")
                pick = hit.argmax(axis=1)
            arr = np.stack([rows + pick, np.minimum(lens, 1)]).astype(np.int32)
            table["_single_gist"] = torch.from_numpy(arr).to(self.device, non_blocking=True)

    def _move_pool_to_host(self, memory: "BatchMemory") -> None:
        """CPU-resident K/V (``kv_cache_residency="cpu"``, ``src/pra_torch/model.py:473-482``): the
        encoded pool moves to pinned host memory (one asynchronous copy on the stream) and the
        device pool is released; the attention kernels then gather only the selected rows over
        the host link (zero-copy), which is the reference's selective host-to-device transfer
        fused into the attention's own row gather.  The gists stay on the device for routing.
        The host buffer is kept by the runtime and reused: only stream-ordered work touches it
        (the next step's copy runs after this step's kernels)."""
        need = memory.pool.numel()
        host = self._host_pool
        if host is None or host.numel() < need:
            if host is not None:
                self._retired_host_pools.append(host)  # never handed back while kernels may read it
            size = 1 << max(need - 1, 1).bit_length()
            host = torch.empty(size, dtype=torch.bfloat16, pin_memory=True)
            self._host_pool = host
        view = host[:need].view(memory.pool.shape)
        view.copy_(memory.pool, non_blocking=True)
        memory.device_kv_bytes = 0
        memory.pool = view
        memory.pools = list(view.unbind(0))

    def _encode_wave(self, memory: BatchMemory, wave_chunks: list[int], first_seq: int, table: dict,
                     packed: torch.Tensor) -> None:
        def view(name, dtype=None):
            off, words, count = table[name]
            t = packed[off: off + words]
            return t.view(torch.uint8)[:count] if dtype == torch.uint8 else t

        n = len(wave_chunks)
        L = memory.seq_len
        ext = _ext.require()
        x = ext.embed_add(view("ids"), None, L, self.tok_emb_w, self.pos_emb_w)
        valid = view("valid", torch.uint8).view(n, L)
        namespace = None
        if table["has_ns"]:
            arrays = [view(name) for name in ("ns0", "ns1", "ns2", "ns3", "ns4", "ns5")]
            namespace = Namespace(table.get("rows_entries"), memory.entries, memory.chunks, self.device, arrays)
            namespace.empty = table["ns_empty"]
        rows = slice(first_seq * L, (first_seq + n) * L)
        hook = None
        if self._single_pass():  # every layer's gists right after its QKV: one pass serves all chunks
            hook = lambda layer: self._pool_gists(memory, table, view, layer)  # noqa: E731
        self.run_blocks(x, n, L, valid, namespace, memory, stop_after_kv=True, pool_rows=rows,
                        budget=view("budget"), query_rows=view("last"), after_qkv=hook)
        if hook is None:
            self._pool_gists(memory, table, view)

    def _pool_gists(self, memory: BatchMemory, table: dict, view, layer: int | None = None) -> None:
        """One launch builds the group's gists for every layer (or for ``layer`` only), written in
        place into the cache tables."""
        cfg = self.cfg
        d = cfg.d_model
        ext = _ext.require()
        pk, pv = memory.k_all(d), memory.v_all(d)
        gk, gv, gn, gc = memory.gist_k_all, memory.gist_v_all, memory.gists_all, memory.gist_count_all
        if layer is not None:
            sel = slice(layer, layer + 1)
            pk, pv, gk, gv, gn, gc = pk[sel], pv[sel], gk[sel], gv[sel], gn[sel], gc[sel]
        start, length, dest = view("gist_rows"), view("lens"), view("dest")
        if cfg.gist_mode in ("last", "ref_end"):  # the mean over one picked row is that row
            start, length = table["_single_gist"][0], table["_single_gist"][1]
        if cfg.gist_mode in ("mean", "last", "ref_end"):
            ext.gist_mean_into(pk, pv, start, length, dest, gk, gv, gn, gc)
            return
        ext.gist_kmeans_into(pk, pv, start, length, dest, gk, gv, gn, gc, table["max_len"], cfg.gist_kmeans_max_iters,
                             float(cfg.gist_kmeans_tol), bool(cfg.gist_kmeans_normalize),
                             cfg.gist_kmeans_init == "kmeans++", cfg.gist_kmeans_empty_cluster_policy == "farthest",
                             view("km_first"), self.kmeans_tables.idx, self.kmeans_tables.draws, view("km_off"), None)

    # -- prompt forward + loss ----------------------------------------------------
    @traced("pra.prompt_forward")
    def prompt_forward(self, input_ids, attention_mask, memory: BatchMemory | None, position_offset=0):
        cfg = self.cfg
        b, t = input_ids.shape
        if torch.is_tensor(position_offset):
            positions = position_offset.to(self.device).view(b, 1) + torch.arange(t, device=self.device)[None]
        else:
            positions = torch.arange(int(position_offset), int(position_offset) + t, device=self.device).expand(b, t)
        if attention_mask is not None:
            positions = positions.masked_fill(~attention_mask.bool(), 0)
        x = self.embed(input_ids, positions)
        valid = attention_mask.to(torch.uint8).contiguous() if attention_mask is not None else None
        namespace = None
        if memory is not None:
            if memory.prompt_ns is not None:
                namespace = Namespace(memory.rows, memory.entries, memory.chunks, self.device, memory.prompt_ns[0])
                namespace.empty = memory.prompt_ns[1]
            else:
                namespace = Namespace(memory.rows, memory.entries, memory.chunks, self.device)
            self.last_namespace = namespace
        budget = cfg.effective_model_max_context_tokens - t - cfg.context_safety_reserve_tokens
        if budget < 0:
            raise ValueError("Direct context and safety reserve exceed model_max_context_tokens.")
        if cfg.max_materialized_memory_tokens is not None:
            budget = min(budget, cfg.max_materialized_memory_tokens)
        last = None
        if attention_mask is not None:
            pos = torch.arange(t, device=self.device).expand(b, t)
            last = pos.masked_fill(~attention_mask.bool(), -1).max(dim=1).values
        self.last_routing = {}
        x = self.run_blocks(x, b, t, valid, namespace, memory, budget=budget, query_rows=last)
        return layer_norm(x, self.ln_f)

    @traced("pra.loss")
    def loss(self, hidden: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        return lm_head_loss(hidden, self.head, labels.reshape(-1).contiguous(), self.cfg.vocab_size, 0)

    def logits(self, hidden: torch.Tensor, b: int, t: int) -> torch.Tensor:
        return lm_head_logits(hidden, self.head)[:, : self.cfg.vocab_size].view(b, t, -1)


class _Unsupported(RuntimeError):
    pass


class _IdsOnlyTokenizer:
    """A tokenizer whose ``decode`` returns an empty string (for partitions whose chunk texts
    are discarded); everything else is the wrapped tokenizer's."""

    def __init__(self, tokenizer):
        self._tokenizer = tokenizer

    def decode(self, ids) -> str:
        return ""

    def __getattr__(self, name):
        return getattr(self._tokenizer, name)


# The prompt's block stack with gradients runs as ONE autograd node over the native
# stack_train_forward / stack_train_backward (the same kernels in the same order as the
# per-layer autograd functions); PRA_TRAIN_STACK=python selects the per-layer path.
_NATIVE_TRAIN_STACK = os.environ.get("PRA_TRAIN_STACK", "native").lower() != "python"
# The native cache-build planner (csrc/planner.cpp); PRA_PLANNER=python keeps the Python planner.
_NATIVE_PLANNER = os.environ.get("PRA_PLANNER", "native").lower() != "python"
# Cache build as one layer-synchronous pass (default) or one full pass per dependency wave.
_LAYER_SYNC = os.environ.get("PRA_CACHE_BUILD", "layer").lower() != "waves"


class _TrainStack(torch.autograd.Function):
    """x [b*t, D] -> the block stack's output; weight gradients land in the flat buffer."""

    @staticmethod
    def forward(ctx, x, rt: "DeviceRuntime", b: int, t: int, key_valid, routing, memory, budget, query_rows):
        cfg = rt.cfg
        d = cfg.d_model
        ext = _ext.require()
        routed = routing is not None and not routing.empty
        ns, gists, counts, gist_kv, budget_rows, settings = [], None, None, None, None, []
        if routed:
            ns = [routing.row_pos_off, routing.row_ref_off, routing.ref_pos_off, routing.pos_chunk, routing.pos_ref,
                  routing.pos_rank, memory.chunk_start, memory.chunk_len, memory.chunk_pool_row]
            gists, counts = memory.gists_all, memory.gist_count_all
            settings, budget_rows = rt._route_settings(budget)
            if cfg.detail_materialization == "gist_only":
                gist_kv = torch.stack([memory.gist_k_all, memory.gist_v_all]).view(
                    2, cfg.n_layers, -1, d).bfloat16()
        mem_pool = memory.pool if routed else None
        out = ext.stack_train_forward(x.contiguous(), b, t, rt._stack_weights(), cfg.n_heads, rt.head_dim, 1e-5,
                                      key_valid, mem_pool, ns, gists, counts, gist_kv, budget_rows, query_rows,
                                      settings)
        n_layers = cfg.n_layers
        _ext.add_launches("stack_train_forward", n_layers * (7 + (1 if routed else 0)))
        pos = 1
        if routed:
            for li in range(n_layers):
                mem_idx, ints, sel_i, sel_f = out[pos: pos + 4]
                rt.last_routing[li] = LayerRouting(mem_idx, ints, sel_i, sel_f)
                pos += 4
        ctx.rt, ctx.b, ctx.t = rt, b, t
        ctx.key_valid, ctx.mem_pool, ctx.gist_kv = key_valid, mem_pool, gist_kv
        ctx.gist_only = bool(routed and settings[6])
        ctx.saved = out[pos:]
        return out[0]

    @staticmethod
    @traced("pra.stack_backward")
    def backward(ctx, dy):
        rt = ctx.rt
        slots = [layer[name] for layer in rt.layers for name in ("ln1", "qkv", "o", "ln2", "up", "down")]
        betas = {s.grad_beta() for s in slots}
        if len(betas) != 1:
            raise RuntimeError("block-stack gradients are partly accumulated: zero_grad between steps")
        empty = torch.empty(0, device=dy.device, dtype=torch.bfloat16)
        grads = []
        for s in slots:
            grads += [s.gw if s.gw is not None else empty, s.gb if s.gb is not None else empty]
        beta = betas.pop()
        ext = _ext.require()
        weights, saved, n_layers = rt._stack_weights(), ctx.saved, rt.cfg.n_layers
        hooks = rt.grad_hooks if beta == 0.0 else None  # (accumulating micro-batches: reduce at the step)
        args = (rt.cfg.n_heads, rt.head_dim, ctx.key_valid)
        if hooks is None:
            dx = ext.stack_train_backward(dy.contiguous(), ctx.b, ctx.t, weights, grads, beta, *args, saved,
                                          ctx.mem_pool, ctx.gist_kv, ctx.gist_only, 0)
        else:
            # layer by layer, so a layer's finished gradients can be reduced across ranks while the
            # layers below it run their backward
            hooks.before_stack()
            dx = dy.contiguous()
            for li in reversed(range(n_layers)):
                dx = ext.stack_train_backward(dx, ctx.b, ctx.t, weights[12 * li: 12 * li + 12],
                                              grads[12 * li: 12 * li + 12], beta, *args,
                                              saved[15 * li: 15 * li + 15], ctx.mem_pool, ctx.gist_kv,
                                              ctx.gist_only, li)
                hooks.after_layer(li)
        ctx.saved = None
        _ext.add_launches("stack_train_backward", 25 * rt.cfg.n_layers)
        return dx, None, None, None, None, None, None, None, None


class _Embed(torch.autograd.Function):
    """x = token_emb[ids] + pos_emb[positions] (bf16); gradients land in the flat buffer."""

    @staticmethod
    def forward(ctx, ids, positions, anchor, rt: DeviceRuntime):
        x = (rt.tok_emb_w[ids].float() + rt.pos_emb_w[positions].float()).bfloat16()
        ctx.rt = rt
        ctx.save_for_backward(ids, positions)
        return x.view(-1, x.shape[-1])

    @staticmethod
    def backward(ctx, dx):
        ids, positions = ctx.saved_tensors
        rt = ctx.rt
        d = dx.shape[-1]
        g = dx.float().view(-1, d)
        tok = torch.zeros(rt.tok_emb_g.shape, device=dx.device, dtype=torch.float32)
        tok.index_add_(0, ids.reshape(-1), g)
        pos = torch.zeros(rt.pos_emb_g.shape, device=dx.device, dtype=torch.float32)
        pos.index_add_(0, positions.reshape(-1), g)
        rt.tok_emb_g.copy_(tok)
        rt.pos_emb_g.copy_(pos)
        return None, None, None, None


# ---------------------------------------------------------------------------
# Model integration
# ---------------------------------------------------------------------------

def attach_device_runtime(model: TinyPRAModel) -> TinyPRAModel:
    reason = unsupported_reason(model.cfg)
    if reason is not None or not _ext.available():
        return model
    runtime = DeviceRuntime(model)
    model._device_runtime = runtime
    model.device_path_enabled = lambda: True
    model.bf16_native = True

    def build_optimizer(train_config):
        return FusedAdamW(runtime.flat, train_config.learning_rate, train_config.weight_decay,
                          max_grad_norm=train_config.max_grad_norm)

    def optimizer_step_hook(optimizer, train_config):
        if isinstance(optimizer, FusedAdamW):
            optimizer.max_grad_norm = train_config.max_grad_norm
            optimizer.step()
            return optimizer.last_norm  # 0-dim device tensor: read it only when it is logged
        raise RuntimeError("device path expects the fused optimizer")

    def announce_batch(batch):
        runtime.upcoming = batch["metadata"] if isinstance(batch, dict) and "metadata" in batch else None

    def prefetch_batch(batch):
        if isinstance(batch, dict) and "metadata" in batch:
            runtime.prefetch(batch["metadata"], part=1, parts=2)  # second half; build_memory plans the rest
            runtime.upcoming = None

    model.build_optimizer = build_optimizer
    model.optimizer_step_hook = optimizer_step_hook
    model.prefetch_batch = prefetch_batch
    model.announce_batch = announce_batch
    model.after_load_state = runtime.flat.refresh_shadow
    original_load = model.load_state_dict

    def load_state_dict(state, strict=True):
        result = original_load(state, strict=strict)
        runtime.flat.refresh_shadow()
        return result

    model.load_state_dict = load_state_dict
    return model


def prepare_model(cfg, device) -> TinyPRAModel:
    """A model on ``device``; on CUDA with a supported config it gets the device runtime."""
    model = TinyPRAModel(cfg).to(device)
    if str(device).startswith("cuda"):
        if not _ext.available():
            raise RuntimeError("CUDA device requested but the pra_ops extension is not built")
        attach_device_runtime(model)
    return model


def device_batch_step(model, batch, device, tokenizer, resolver_config, cache_config):
    """Device version of the PRA batch step: batched cache build, one prompt forward, fused loss."""
    rt: DeviceRuntime = model._device_runtime
    metadata = batch["metadata"]
    t0 = time.perf_counter()
    try:
        memory, caches, builders = rt.build_memory(metadata, tokenizer, resolver_config)
    except _Unsupported:
        model.device_path_enabled = lambda: False
        from ..pra_train import _pra_batch_step

        return _pra_batch_step(model, batch, device, tokenizer, resolver_config, cache_config)
    build_s = time.perf_counter() - t0
    ids = batch["input_ids"].to(device, non_blocking=True)
    mask = batch["attention_mask"].to(device, non_blocking=True)
    labels = batch["labels"].to(device, non_blocking=True)
    hidden = rt.prompt_forward(ids, mask, memory if memory.chunks else None)
    loss = rt.loss(hidden, labels)
    if rt.upcoming is not None:  # first half of the next batch's host planning overlaps this forward
        rt.prefetch(rt.upcoming, part=0, parts=2)
    # a device mask's token count stays on the device (read lazily, after the step's loss read)
    am = batch["attention_mask"]
    tokens = int(am.sum()) if am.device.type == "cpu" else am.sum()
    b = ids.shape[0]
    metrics = {"cache_build_duration_seconds": build_s / max(b, 1), "cache_build_total_duration_seconds": build_s,
               "logical_batch_size": float(b), "prompt_forward_calls": 1.0,
               "cached_kv_bytes": float(memory.kv_bytes), "gpu_cached_kv_bytes": float(memory.device_kv_bytes)}
    return loss, {"tokens": tokens, "examples": b, "batch": batch, "caches": caches, "metrics": metrics,
                  "memory": memory, "hidden": hidden}


def pra_attention_device(layer, x, attention_mask):
    raise RuntimeError("per-layer device attention is driven by DeviceRuntime.run_blocks")


# ---------------------------------------------------------------------------
# Self-test of the routing kernel against the object path (used by the GPU tests)
# ---------------------------------------------------------------------------

def routing_selftest(device, seed: int = 0) -> None:
    """Random namespaces routed on the device and through ``PRASimpleMemoryCache`` + budget."""
    from ..config import PRAConfig
    from ..memory.cache import (ChunkRoutingGist, LayerKV, LayerReferenceMemory, PRACacheEntry,
                                PRASimpleMemoryCache, ReferenceChunkMemory)
    from .attention import budget_selection

    gen = torch.Generator().manual_seed(seed)
    d, g_max = 64, 2
    cfg = PRAConfig(d_model=d, n_heads=2, top_k_references=2, top_k_chunks_per_reference=3, trigger_threshold=-0.5,
                    max_seq_len=400, gist_mode="kmeans", gists_per_chunk=g_max)
    rows, entries, chunks = [], [], []
    caches = []
    for row in range(3):
        cache = PRASimpleMemoryCache()
        row_entries = []
        for r in range(4 + row):
            uri = f"mem://row{row}/doc{(r * 5) % 7}"
            e = len(entries)
            rec = EntryRecord(row, uri, "", {}, False, ())
            entry = PRACacheEntry(uri=uri, text="")
            mem = LayerReferenceMemory()
            for c in range(1 + (r * 3 + row) % 12):
                n = 10 + (c * 7) % 30
                gist = torch.randn(1 + c % g_max, d, generator=gen)
                ci = len(chunks)
                chunks.append(ChunkRecord(row, e, uri, f"{uri}#chunk={c}", c * 40, c * 40 + n, tuple(range(n)),
                                          seq=ci))
                rec.chunks.append(ci)
                kv = torch.zeros(1, 2, n, d // 2)
                mem.chunks.append(ReferenceChunkMemory(f"{uri}#chunk={c}", uri, c * 40, c * 40 + n, LayerKV(kv, kv),
                                                       ChunkRoutingGist(k=gist)))
                chunks[ci].metadata["gist"] = gist
            entry.layer_memory[0] = mem
            cache.put(entry)
            entries.append(rec)
            row_entries.append(e)
        caches.append(cache)
        rows.append(row_entries)
    seq_len = 64
    ns = Namespace(rows, entries, chunks, device)
    C = len(chunks)
    gists = torch.zeros(C, g_max, d)
    counts = torch.zeros(C, dtype=torch.int32)
    for i, c in enumerate(chunks):
        k = c.metadata["gist"]
        gists[i, : k.shape[0]] = torch.nn.functional.normalize(k, dim=-1, eps=1e-12)
        counts[i] = k.shape[0]
    query = torch.randn(3, d, generator=gen)
    t = 120
    budget = cfg.effective_model_max_context_tokens - t
    as_int = lambda x: torch.tensor(x, dtype=torch.int32, device=device)  # noqa: E731
    mem_idx, ints, sel_i, sel_f = _ext.require().route(
        query.bfloat16().to(device), gists.to(device), counts.to(device), ns.row_pos_off, ns.row_ref_off,
        ns.ref_pos_off, ns.pos_chunk, ns.pos_ref, ns.pos_rank, as_int([c.token_start for c in chunks]),
        as_int([len(c.token_ids) for c in chunks]), as_int([c.seq * seq_len for c in chunks]), cfg.top_k_references,
        cfg.top_k_chunks_per_reference, 0, 0, float(cfg.trigger_threshold), budget, False, False, True, 16, budget,
        None, None)
    mem_idx, ints, sel_i, sel_f = mem_idx.cpu(), ints.cpu(), sel_i.cpu(), sel_f.cpu()
    q_bf = query.bfloat16().float()
    for row in range(3):
        hits = caches[row].search(q_bf[row:row + 1], 0, cfg)[0]
        hits = [h for h in hits if h.chunk_score >= cfg.trigger_threshold]
        kept, _ = budget_selection(hits, cfg, direct_tokens=t, routing_candidates=len(hits))
        device_chunks = [chunks[int(c)].chunk_id for c in sel_i[0, row, : int(ints[1, row])]]
        assert sorted(device_chunks) == sorted(h.chunk_id for h in kept), (row, device_chunks,
                                                                           [h.chunk_id for h in kept])
        expected_rows = []
        for h in sorted(kept, key=lambda s: (s.reference_uri, s.token_start, s.chunk_id)):
            ci = next(i for i, c in enumerate(chunks) if c.chunk_id == h.chunk_id and c.row == row)
            expected_rows += [chunks[ci].seq * seq_len + j for j in range(len(chunks[ci].token_ids))]
        got = mem_idx[row, : int(ints[0, row])].tolist()
        assert got == expected_rows, (row, got[:10], expected_rows[:10])
        for j, h in enumerate(sorted(kept, key=lambda s: (-s.chunk_score, s.reference_uri, s.chunk_id))):
            assert math.isfinite(float(sel_f[1, row, j]))
