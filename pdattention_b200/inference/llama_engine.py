"""Device inference engine for the PRA Llama-family models (prefill + decode on sm_100a kernels).

Layout on one GPU (tensor parallelism shards the head / column dimensions, see
``pdattention_b200.parallel.tp``):

* weights (bf16): per layer a fused ``[q | k | v]`` projection (+ Qwen2 biases), the
  output projection, a fused ``[gate | up]`` projection and the down projection;
* chunk memory (``ChunkMemory``): per layer one pool ``[rows, 2 * kv_dim]`` holding the
  post-rotary keys and the values of every reference token (chunk c owns rows
  ``row0[c] .. row0[c] + len[c]``), plus the routing gists (mean pre-rotary key per
  chunk) in fp32 (exact rescoring) and bf16 (tensor-core scoring);
* local KV cache: per layer ``[2, B, max_len, kv_dim]`` for the direct window and the
  generated tokens.

Per layer and step: RMSNorm -> QKV GEMM -> routing (tensor-core scores + exact
top-k) -> rotary copy of q in place and of k/v into the cache -> attention over
[selected memory ; local causal] -> O GEMM with the residual fused -> RMSNorm ->
gate/up GEMM -> SwiGLU -> down GEMM with the residual fused.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from ..models.llama import PRALlamaConfig, PRALlamaReference
from ..ops import _ext
from ..tracing import traced
from .routing import select_chunks

# Decode projections on this library's decode GEMM (PRA_DECODE_GEMM=cutlass keeps the CUTLASS
# stream-K GEMM and the separate all-reduce); rows per call it serves.
_DECODE_GEMM = os.environ.get("PRA_DECODE_GEMM", "native").lower() != "cutlass"
_DECODE_ROWS = 64


# ---------------------------------------------------------------------------
# Weights
# ---------------------------------------------------------------------------

@dataclass
class LayerWeights:
    ln_in: torch.Tensor
    qkv: torch.Tensor          # [q_dim + 2 kv_dim (local shard), d]
    qkv_bias: torch.Tensor | None
    o: torch.Tensor            # [d, q_dim (local shard)]
    ln_post: torch.Tensor
    gate_up: torch.Tensor      # [2 F (local shard), d]
    down: torch.Tensor         # [d, F (local shard)]
    qkv_route: torch.Tensor | None = None       # [q | k | v | routing-query rows] (decode GEMM)
    qkv_route_bias: torch.Tensor | None = None


class LlamaWeights:
    """bf16 device weights (optionally one tensor-parallel shard)."""

    def __init__(self, cfg: PRALlamaConfig, layers: list[LayerWeights], embed: torch.Tensor, norm: torch.Tensor,
                 head: torch.Tensor, tp_rank: int = 0, tp_size: int = 1):
        self.cfg, self.layers, self.embed, self.norm, self.head = cfg, layers, embed, norm, head
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.mlp_block = 0  # > 0: gate / up rows interleaved in runs of this many (set by an engine)
        self.norm_folded = False  # RMSNorm weights multiplied into qkv_route / gate_up (set by an engine)
        self.route_rows = False  # routing-query rows appended to every QKV weight (set by an engine)

    @staticmethod
    def _shard_rows(t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
        n = t.shape[0] // size
        return t[rank * n:(rank + 1) * n]

    @classmethod
    def from_reference(cls, model: PRALlamaReference, device, tp_rank: int = 0, tp_size: int = 1) -> "LlamaWeights":
        cfg = model.cfg
        if cfg.num_key_value_heads % tp_size or cfg.intermediate_size % tp_size:
            raise ValueError("tensor-parallel size must divide the KV heads and the MLP width")
        dev = torch.device(device)
        bf = lambda t: t.detach().to(dev, torch.bfloat16).contiguous()  # noqa: E731
        rows = cls._shard_rows
        layers = []
        for layer in model.model.layers:
            a, m = layer.self_attn, layer.mlp
            q = rows(a.q_proj.weight, tp_rank, tp_size)
            k = rows(a.k_proj.weight, tp_rank, tp_size)
            v = rows(a.v_proj.weight, tp_rank, tp_size)
            bias = None
            if cfg.attention_bias:
                bias = bf(torch.cat([rows(a.q_proj.bias, tp_rank, tp_size), rows(a.k_proj.bias, tp_rank, tp_size),
                                     rows(a.v_proj.bias, tp_rank, tp_size)]))
            o = a.o_proj.weight.t().contiguous()
            layers.append(LayerWeights(
                ln_in=bf(layer.input_layernorm.weight), qkv=bf(torch.cat([q, k, v])), qkv_bias=bias,
                o=bf(rows(o, tp_rank, tp_size).t()), ln_post=bf(layer.post_attention_layernorm.weight),
                gate_up=bf(torch.cat([rows(m.gate_proj.weight, tp_rank, tp_size),
                                      rows(m.up_proj.weight, tp_rank, tp_size)])),
                down=bf(rows(m.down_proj.weight.t().contiguous(), tp_rank, tp_size).t())))
        head = model.head_weight()
        return cls(cfg, layers, bf(model.model.embed_tokens.weight), bf(model.model.norm.weight), bf(head),
                   tp_rank, tp_size)

    @classmethod
    def random(cls, cfg: PRALlamaConfig, device, seed: int = 0, std: float = 0.02, tp_rank: int = 0,
               tp_size: int = 1) -> "LlamaWeights":
        """Random-init weights generated directly on the device (8B-class models)."""
        dev = torch.device(device)
        gen = torch.Generator(device=dev).manual_seed(seed + 1000 * tp_rank)

        def rand(*shape):
            return (torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32) * std).to(torch.bfloat16)

        d, f = cfg.hidden_size, cfg.intermediate_size // tp_size
        qd, kd = cfg.q_dim // tp_size, cfg.kv_dim // tp_size
        ones = lambda: torch.ones(d, device=dev, dtype=torch.bfloat16)  # noqa: E731
        layers = [LayerWeights(ln_in=ones(), qkv=rand(qd + 2 * kd, d),
                               qkv_bias=rand(qd + 2 * kd) if cfg.attention_bias else None, o=rand(d, qd),
                               ln_post=ones(), gate_up=rand(2 * f, d), down=rand(d, f))
                  for _ in range(cfg.num_hidden_layers)]
        gen_shared = torch.Generator(device=dev).manual_seed(seed)  # embeddings / head replicated
        embed = (torch.randn(cfg.vocab_size, d, generator=gen_shared, device=dev) * std).to(torch.bfloat16)
        head = embed if cfg.tie_word_embeddings else \
            (torch.randn(cfg.vocab_size, d, generator=gen_shared, device=dev) * std).to(torch.bfloat16)
        return cls(cfg, layers, embed, ones(), head, tp_rank, tp_size)


# ---------------------------------------------------------------------------
# Chunk memory
# ---------------------------------------------------------------------------

class ChunkMemory:
    """Per-layer chunk K/V pools and routing gists on the device."""

    def __init__(self, cfg: PRALlamaConfig, n_chunks: int, kv_dim: int, device, chunk_tokens: int | None = None,
                 gist_dim: int | None = None):
        self.cfg = cfg
        self.C = n_chunks
        self.C_pad = (n_chunks + 7) // 8 * 8  # score rows stay 32-byte aligned for the scoring GEMM
        self.tc = chunk_tokens or cfg.chunk_tokens
        self.kv_dim = kv_dim                  # K/V width held here (this rank's KV heads)
        self.gist_dim = gist_dim or kv_dim    # routing width (every KV head: gists are replicated)
        L = cfg.num_hidden_layers
        dev = torch.device(device)
        self.pool = torch.empty((L, n_chunks * self.tc, 2 * kv_dim), device=dev, dtype=torch.bfloat16)
        # gist tables [3, L, C, 1, gist_dim]: routing copy (normalised), key mean, value mean (unused)
        self.tables = torch.zeros((3, L, self.C_pad, 1, self.gist_dim), device=dev, dtype=torch.float32)
        self.gn, self.gk, self.gv = self.tables.unbind(0)
        self.gn_bf16 = torch.zeros((L, self.C_pad, self.gist_dim), device=dev, dtype=torch.bfloat16)
        self.count = torch.zeros((L, self.C_pad), device=dev, dtype=torch.int32)
        self.chunk_len = torch.zeros(self.C_pad, device=dev, dtype=torch.int32)
        self.chunk_row0 = (torch.arange(self.C_pad, device=dev, dtype=torch.int32) * self.tc)

    def k(self, layer: int) -> torch.Tensor:
        return self.pool[layer][:, : self.kv_dim]

    def v(self, layer: int) -> torch.Tensor:
        return self.pool[layer][:, self.kv_dim:]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.pool, self.tables, self.gn_bf16))


# ---------------------------------------------------------------------------
# Engine
# ---------------------------------------------------------------------------

class PRALlamaEngine:
    """Batched prefill / decode of a PRA Llama-family model on one GPU (or one TP shard)."""

    def __init__(self, weights: LlamaWeights, device, tp=None, decode_split_keys: int | None = None,
                 k_cand_factor: int = 4,
                 shard_routing: bool = True, kv_residency: str = "gpu", overlap_routing: bool | None = None):
        self.w = weights
        self.cfg = weights.cfg
        self.device = torch.device(device)
        self.tp = tp  # tensor-parallel communicator (None: one GPU)
        cfg = self.cfg
        self.tp_size = weights.tp_size
        self.heads = cfg.num_attention_heads // self.tp_size
        self.kv_heads = cfg.num_key_value_heads // self.tp_size
        self.q_dim = self.heads * cfg.head_dim
        self.kv_dim = self.kv_heads * cfg.head_dim
        self.split_keys = decode_split_keys  # None: chosen per step from the grid it gives
        self.k_cand_factor = k_cand_factor
        self.shard_routing = shard_routing  # TP: score chunk slices per rank + cross-GPU top-k merge
        if kv_residency not in ("gpu", "cpu"):
            raise ValueError("kv_residency must be 'gpu' or 'cpu'")
        # "cpu": the chunk K/V pool lives in pinned host memory after the build; routing stays
        # on the device (gists) and the attention kernels gather only the selected rows over the
        # host link (a memory larger than the GPU's HBM at the cost of link bandwidth per step)
        self.kv_residency = kv_residency
        # Decode: the local-window attention splits run on the current stream while routing and
        # the memory splits run on a high-priority side stream (PRA_ROUTE_OVERLAP=0: serial).
        if overlap_routing is None:
            overlap_routing = os.environ.get("PRA_ROUTE_OVERLAP", "1") != "0"
        self.overlap_routing = overlap_routing and self.device.type == "cuda"
        self._route_stream: torch.cuda.Stream | None = None
        self._parts: tuple[tuple[int, int], torch.Tensor, torch.Tensor] | None = None
        self._bounds_cache: tuple | None = None
        # overlapped decode: the local-window splits run as a persistent grid of this many CTAs
        # (default two per SM) so every SM keeps a slot for the routing chain and memory splits
        self._local_ctas = int(os.environ.get("PRA_LOCAL_CTAS", "-1"))
        self.ext = _ext.require()
        self._rope_cache: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.memory: ChunkMemory | None = None
        self.cache: torch.Tensor | None = None
        self.cache_len: torch.Tensor | None = None
        self.namespace: tuple[torch.Tensor, torch.Tensor] | None = None
        self.page_table: torch.Tensor | None = None  # [B, P] pages per row (paged chunk cache)
        self._row0 = 0  # first row of the prefill row batch being routed
        self.last_selection: dict[int, torch.Tensor] = {}
        # Vocabulary-parallel LM head: under tensor parallelism each rank holds rows
        # [vocab_start, vocab_end) of the head and computes only that slice of the logits.
        vocab = self.w.head.shape[0]
        per = -(-vocab // self.tp_size)
        per = -(-per // 8) * 8  # 16-byte aligned slices
        rank = self.w.tp_rank
        self.vocab_start = min(vocab, rank * per)
        self.vocab_end = min(vocab, self.vocab_start + per)
        self.head_local = self.w.head[self.vocab_start: self.vocab_end]
        # Decode (<= 64 rows) runs its projections on this library's decode GEMM, the row-parallel
        # ones fused with their all-reduce; each layer's QKV weight gains the routing-query rows.
        self.native_decode = _DECODE_GEMM
        self.route_dim = cfg.num_key_value_heads * cfg.head_dim
        self._ones = torch.ones(cfg.hidden_size, device=self.device, dtype=torch.bfloat16)
        self._ss_tiles = cfg.hidden_size // 128
        self._ss: torch.Tensor | None = None  # [2, hidden / 128, 64] folded-norm sums of squares
        if self.native_decode:
            self._attach_route_rows()

    def _attach_route_rows(self) -> None:
        """Append to every layer's ``[q | k | v]`` weight the routing-query rows: for each KV head,
        the mean of its group's query rows (over ALL ranks' heads, gathered once here), so the
        decode QKV GEMM also yields the full-width routing query (the KV-group mean of the
        pre-rotary query) and routing needs no per-step gather.  ``lw.qkv`` becomes a view of the
        first rows (no second copy of the projection)."""
        cfg = self.cfg
        g, dh = cfg.group, cfg.head_dim
        qd, kd = self.q_dim, self.kv_dim
        if getattr(self.w, "route_rows", False):  # once per weight set (engines may share one)
            self._block_mlp_rows()
            self._fold_norms()
            return

        def group_mean(rows: torch.Tensor) -> torch.Tensor:  # [heads * dh, ...] -> [kv_heads * dh, ...]
            return rows.float().unflatten(0, (self.kv_heads, g, dh)).mean(1).flatten(0, 1)

        def gather(t: torch.Tensor) -> torch.Tensor:
            if self.tp is None:
                return t
            import torch.distributed as dist

            parts = [torch.empty_like(t) for _ in range(self.tp_size)]
            dist.all_gather(parts, t.contiguous(), group=self.tp.group)
            return torch.cat(parts)  # rank-major = KV-head order

        for lw in self.w.layers:
            route = gather(group_mean(lw.qkv[:qd]).to(torch.bfloat16))
            fused = torch.cat([lw.qkv, route]).contiguous()
            lw.qkv_route = fused
            lw.qkv = fused[: qd + 2 * kd]
            lw.qkv_route_bias = None
            if lw.qkv_bias is not None:
                rb = gather(group_mean(lw.qkv_bias[:qd]).to(torch.bfloat16))
                lw.qkv_route_bias = torch.cat([lw.qkv_bias, rb]).contiguous()
                lw.qkv_bias = lw.qkv_route_bias[: qd + 2 * kd]
        self.w.route_rows = True
        self._block_mlp_rows()
        self._fold_norms()

    def _fold_norms(self) -> None:
        """Multiply each layer's RMSNorm weights into the columns of the projection after them
        (``qkv_route`` <- ``ln_in``, ``gate_up`` <- ``ln_post``), once per weight set.  The decode
        GEMMs then apply the norm as one row scale in their epilogue (the sums of squares come
        from the GEMM that produced the residual stream), and every explicit RMSNorm (prefill,
        chunk encoding, batches above 64 rows) normalises with unit weights."""
        if getattr(self.w, "norm_folded", False) or self.cfg.hidden_size % 128:
            return
        qd, kd = self.q_dim, self.kv_dim
        for lw in self.w.layers:
            fused = (lw.qkv_route.float() * lw.ln_in.float()[None, :]).to(torch.bfloat16).contiguous()
            lw.qkv_route = fused
            lw.qkv = fused[: qd + 2 * kd]
            lw.gate_up = (lw.gate_up.float() * lw.ln_post.float()[None, :]).to(torch.bfloat16).contiguous()
        self.w.norm_folded = True

    def _block_mlp_rows(self, block: int = 64) -> None:
        """Interleave every layer's ``[gate | up]`` rows in runs of ``block`` (``[gate 0..63 |
        up 0..63 | gate 64..127 | ...]``), once per weight set: a 128-row tile of the decode GEMM then
        holds matching gate and up features and applies SwiGLU in its epilogue; larger batches
        use the same layout through ``silu_mul(..., block)``."""
        if getattr(self.w, "mlp_block", 0) or not self.native_decode:
            return
        f = self.w.layers[0].gate_up.shape[0] // 2
        if f % block:
            return
        for lw in self.w.layers:
            d = lw.gate_up.shape[1]
            g, u = lw.gate_up[:f].view(f // block, block, d), lw.gate_up[f:].view(f // block, block, d)
            lw.gate_up = torch.stack([g, u], 1).reshape(2 * f, d).contiguous()
        self.w.mlp_block = block

    # -- helpers ----------------------------------------------------------------
    def rope_tables(self, max_pos: int) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 cos/sin ``[max_pos, Dh/2]`` computed in fp64 (cached, grown on demand)."""
        have = max(self._rope_cache) if self._rope_cache else 0
        if have < max_pos:
            cfg = self.cfg
            n = max(max_pos, 2 * have)
            half = cfg.head_dim // 2
            inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, half, dtype=torch.float64) / half))
            ang = torch.arange(n, dtype=torch.float64)[:, None] * inv[None]
            self._rope_cache = {n: (ang.cos().float().to(self.device), ang.sin().float().to(self.device))}
        return next(iter(self._rope_cache.values()))

    def _norm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return self.ext.norm_fwd(x, w, None, self.cfg.rms_norm_eps, True)[0]

    def _split_for(self, rows: int, max_keys: int) -> int:
        """Keys per decode-attention split: the longest split (1024 measured best on the full-size
        layer: 0.92 of the HBM copy rate) whose grid still fills three CTAs per SM, else the
        shortest (more CTAs for the small per-rank work of wide tensor parallelism)."""
        if self.split_keys is not None:
            return self.split_keys
        slots = 3 * torch.cuda.get_device_properties(self.device).multi_processor_count
        for split in (1024, 512):
            if rows * self.kv_heads * -(-max_keys // split) >= slots:
                return split
        return 256

    def _decode_rows(self, x) -> bool:
        return self.native_decode and x.shape[0] <= _DECODE_ROWS

    def _gemm(self, x, w, bias=None, residual=None, ss_out=None) -> torch.Tensor:
        out = torch.empty((x.shape[0], w.shape[0]), device=x.device, dtype=torch.bfloat16)
        if self._decode_rows(x):
            self.ext.decode_gemm(x, w, bias, residual, out, None, 0, 0, [], [], 0, None, 0, None, ss_out=ss_out)
            return out
        self.ext.gemm("tn", x, w, residual, out, bias, None, 1.0, 1.0 if residual is not None else 0.0, None)
        return out

    def _row_parallel(self, x, w, residual, ss_out=None) -> torch.Tensor:
        """out = residual + x @ w^T, summed over tensor-parallel ranks (decode rows: one fused
        GEMM + all-reduce kernel).  ``ss_out`` (decode rows): the output's per-tile row sums of
        squares for the next, folded RMSNorm."""
        if self.tp is None:
            return self._gemm(x, w, residual=residual, ss_out=ss_out)
        if self._decode_rows(x) and x.shape[0] <= self.tp.decode_rows and w.shape[0] <= self.tp.decode_width:
            return self.tp.fused_gemm_allreduce(x, w, residual, ss_out=ss_out)
        return self.tp.gemm_allreduce(x, w, residual)

    def _mlp(self, lw: LayerWeights, x: torch.Tensor, ss=None) -> torch.Tensor:
        """SwiGLU MLP with its residual.  ``ss`` (decode rows, folded norms): ``(ss_in, ss_out)``,
        the per-tile sums of squares of ``x`` (its RMSNorm, folded into ``gate_up``) and where the
        down projection leaves those of its output (the next layer's input norm)."""
        blocked = getattr(self.w, "mlp_block", 0)
        act = torch.empty((x.shape[0], lw.gate_up.shape[0] // 2), device=x.device, dtype=torch.bfloat16)
        if ss is not None:
            # one GEMM: the folded post-attention RMSNorm, SwiGLU in the epilogue
            norm = dict(ss_in=ss[0], ss_tiles=self._ss_tiles, ss_dim=self.cfg.hidden_size, ss_eps=self.cfg.rms_norm_eps)
            if blocked == 64 and lw.gate_up.shape[0] % 128 == 0:
                self.ext.decode_gemm(x, lw.gate_up, None, None, act, None, 0, 0, [], [], 0, None, 0, None,
                                     swiglu=True, **norm)
            else:
                gu = torch.empty((x.shape[0], lw.gate_up.shape[0]), device=x.device, dtype=torch.bfloat16)
                self.ext.decode_gemm(x, lw.gate_up, None, None, gu, None, 0, 0, [], [], 0, None, 0, None, **norm)
                self.ext.silu_mul(gu, act, blocked)
            return self._row_parallel(act, lw.down, x, ss_out=ss[1])
        h = self._norm(x, self._ln(lw.ln_post))
        if blocked == 64 and self._decode_rows(h) and lw.gate_up.shape[0] % 128 == 0:
            # one GEMM: SwiGLU in the epilogue of the [gate | up]-interleaved weight
            self.ext.decode_gemm(h, lw.gate_up, None, None, act, None, 0, 0, [], [], 0, None, 0, None, swiglu=True)
        else:
            gu = self._gemm(h, lw.gate_up)
            self.ext.silu_mul(gu, act, blocked)
        return self._row_parallel(act, lw.down, x)

    def _ln(self, weight: torch.Tensor) -> torch.Tensor:
        """The weight an explicit RMSNorm applies: ones once the norm weights are folded into
        the projections after them."""
        return self._ones if getattr(self.w, "norm_folded", False) else weight

    def _embed(self, ids: torch.Tensor) -> torch.Tensor:
        return self.w.embed[ids.reshape(-1)].contiguous()

    def _route(self, layer: int, q_rows: torch.Tensor | None, rows: int, namespace=None,
               route_query: torch.Tensor | None = None):
        """Routing query (group mean of the pre-rotary query) -> memory row lists.

        ``route_query`` is that query already at full width (bf16, from the decode QKV GEMM);
        without it the mean is taken here from this rank's query heads and gathered.  Scores
        against the normalised gists only rank the chunks (a query's norm is the same for all
        of them); the candidates are rescored as exact fp32 cosines."""
        cfg, mem = self.cfg, self.memory
        if route_query is not None:
            rqn = route_query
            rq = route_query  # bf16: the routing kernel widens it while staging it in shared memory
        else:
            rq = q_rows.float().view(rows, self.kv_heads, cfg.group, cfg.head_dim).mean(2).reshape(rows, self.kv_dim)
            if self.tp is not None:
                rq = self.tp.all_gather_columns(rq)  # full kv_dim routing query on every rank
            rqn = torch.nn.functional.normalize(rq, dim=-1, eps=1e-12).to(torch.bfloat16)
        k = cfg.top_k_chunks
        k_cand = min(max(k * self.k_cand_factor, k), 512)
        budget = cfg.memory_budget_tokens if cfg.memory_budget_tokens is not None else -1
        mem_max = cfg.memory_tokens_per_row
        start, end = namespace if namespace is not None else self.namespace
        gn = mem.gn[layer].view(mem.C_pad, -1)
        pages = self.page_table
        if pages is not None and namespace is not None and pages.shape[0] != rows:
            pages = pages[self._row0: self._row0 + rows].contiguous()  # a prefill row batch
        shards = self.tp.world if (self.tp is not None and self.shard_routing and pages is None) else 1
        if shards == 1:
            scores = torch.empty((rows, mem.C_pad), device=self.device, dtype=torch.float32)
            self._score(rqn, mem.gn_bf16[layer], scores)
            mem_idx, mem_len, sel = select_chunks(self.ext, scores, rq, gn, start, end, mem.chunk_len,
                                                  mem.chunk_row0, k, k_cand, budget, mem_max,
                                                  pool_rows=mem.pool.shape[1], page_table=pages)
        else:
            # chunk-sharded routing: this rank scores its slice of the chunks, keeps its exact
            # local top-k, and the ranks' candidates are all-gathered and merged
            c0, c1 = self._route_slice(mem)
            width = c1 - c0
            scores = torch.empty((rows, width), device=self.device, dtype=torch.float32)
            self._score(rqn, mem.gn_bf16[layer][c0:c1], scores)
            lo, hi = self._slice_bounds(start, end, c0, width)
            mem_idx, mem_len, sel = select_chunks(self.ext, scores, rq, gn[c0:c1], lo, hi, mem.chunk_len,
                                                  mem.chunk_row0, k, k_cand, budget, mem_max, id_offset=c0,
                                                  comm=self.tp, global_len=mem.chunk_len,
                                                  global_row0=mem.chunk_row0, pool_rows=mem.pool.shape[1])
        self.last_selection[layer] = sel
        return mem_idx, mem_len

    def _score(self, rqn: torch.Tensor, gists: torch.Tensor, scores: torch.Tensor) -> None:
        """fp32 query x gist scores.  Decode rows use the tcgen05 decode GEMM with a 2-stage ring:
        its CTAs fit beside the local-window attention CTAs they overlap with (a persistent
        library-style GEMM needs a whole SM and waits for the attention to drain one)."""
        if self._decode_rows(rqn) and gists.shape[1] % 64 == 0 and gists.shape[0] % 8 == 0:
            self.ext.decode_gemm(rqn, gists, None, None, scores, None, 0, 0, [], [], 0, None, 0, None)
        else:
            self.ext.gemm("tn_f32", rqn, gists, None, scores, None, None, 1.0, 0.0, None)

    def _slice_bounds(self, start: torch.Tensor, end: torch.Tensor, c0: int, width: int):
        """Each row's namespace clipped to this rank's chunk slice, as slice-local int32 bounds.
        Computed once per (namespace, slice) and kept: the decode steps of a batch share it (a
        new namespace is a new pair of tensors from ``set_namespace``)."""
        key = (start.data_ptr(), end.data_ptr(), start.numel(), end.numel(), start._version, end._version, c0, width)
        cached = self._bounds_cache
        if cached is None or cached[0] != key:
            lo = (start - c0).clamp(0, width).to(torch.int32)
            hi = (end - c0).clamp(0, width).to(torch.int32)
            self._bounds_cache = cached = (key, lo, hi, start, end)  # holds the inputs: their addresses stay theirs
        return cached[1], cached[2]

    def _route_slice(self, mem) -> tuple[int, int]:
        """This rank's chunk slice for sharded routing (8-aligned, covers the padded table)."""
        per = (mem.C_pad // self.tp.world + 7) // 8 * 8
        c0 = min(mem.C_pad, self.tp.rank * per)
        return c0, min(mem.C_pad, c0 + per)

    # -- memory build -----------------------------------------------------------------
    @torch.no_grad()
    @traced("pra.llama.build_memory")
    def build_memory(self, chunks: torch.Tensor, lengths: torch.Tensor, batch_chunks: int = 256) -> ChunkMemory:
        """Encode ``chunks`` ``[C, Tc]`` (each its own sequence from position 0) into a
        ``ChunkMemory`` (for tensor parallelism: this rank's KV heads of every chunk)."""
        cfg = self.cfg
        C, tc = chunks.shape
        mem = ChunkMemory(cfg, C, self.kv_dim, self.device, tc, gist_dim=cfg.kv_dim)
        self.encode_into(mem, chunks, lengths, 0, batch_chunks)
        if self.kv_residency == "cpu":
            host = torch.empty(mem.pool.shape, dtype=mem.pool.dtype, pin_memory=True)
            host.copy_(mem.pool, non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()  # the device pool is released next
            mem.pool = host
        self.memory = mem
        return mem

    @torch.no_grad()
    def encode_into(self, mem: ChunkMemory, chunks: torch.Tensor, lengths: torch.Tensor, first: int,
                    batch_chunks: int = 256) -> None:
        """Encode ``chunks`` ``[n, Tc]`` into chunk slots ``first .. first + n`` of ``mem`` (K/V pool
        rows, gists and their bf16 routing copy, lengths); slots outside are untouched."""
        cfg = self.cfg
        n, tc = chunks.shape
        if n == 0:
            return
        mem.chunk_len[first: first + n].copy_(lengths.to(self.device, torch.int32))
        cos, sin = self.rope_tables(tc)
        if self.tp is not None:  # each row-parallel partial must fit the peer buffer
            batch_chunks = max(1, min(batch_chunks, self.tp.max_partial // (tc * cfg.hidden_size)))
        for c0 in range(0, n, batch_chunks):
            c1 = min(n, c0 + batch_chunks)
            self._encode_chunk_batch(mem, chunks[c0:c1].to(self.device), mem.chunk_len[first + c0: first + c1],
                                     first + c0, cos, sin)
        if self.tp is not None:  # gists are computed per KV-head slice; every rank gets all of them
            self.tp.gather_gists(mem, first, n)
        # bf16 routing copy for the tensor-core scoring GEMM
        sl = slice(first, first + n)
        mem.gn_bf16[:, sl].copy_(mem.gn.view(cfg.num_hidden_layers, mem.C_pad, -1)[:, sl])

    def _encode_chunk_batch(self, mem: ChunkMemory, ids, lengths, c0, cos, sin):
        cfg, ext = self.cfg, self.ext
        n, tc = ids.shape
        M = n * tc
        pos = torch.arange(tc, device=self.device, dtype=torch.int32).repeat(n)
        rows = (torch.arange(M, device=self.device, dtype=torch.int32) + c0 * tc)
        valid = (torch.arange(tc, device=self.device)[None] < lengths[:, None]).to(torch.uint8).contiguous()
        dest = torch.arange(c0, c0 + n, device=self.device, dtype=torch.int32)
        starts = rows.view(n, tc)[:, 0].contiguous()
        x = self._embed(ids)
        qd, kd = self.q_dim, self.kv_dim
        for li, lw in enumerate(self.w.layers):
            h = self._norm(x, self._ln(lw.ln_in))
            qkv = self._gemm(h, lw.qkv, lw.qkv_bias)
            # gist: mean pre-rotary key of each chunk
            k_pre = qkv[:, qd: qd + kd]
            pool = mem.pool[li]
            gk, gv, gn = (mem.gk[li: li + 1], mem.gv[li: li + 1], mem.gn[li: li + 1]) if self.tp is None else \
                self.tp.local_gist_tables(mem, li)
            ext.gist_mean_into(k_pre, qkv[:, qd + kd: qd + 2 * kd], starts - c0 * tc, lengths, dest, gk, gv, gn,
                               mem.count[li: li + 1])
            ext.rope_copy(k_pre, pool[:, :kd], rows, pos, cos, sin, self.kv_heads, cfg.head_dim)
            ext.rope_copy(qkv[:, qd + kd:], pool[:, kd:], rows, None, None, None, self.kv_heads, cfg.head_dim)
            ext.rope_copy(qkv[:, :qd], qkv[:, :qd], None, pos, cos, sin, self.heads, cfg.head_dim)
            if li == len(self.w.layers) - 1:
                break  # the last layer's output is never read
            kv = pool[c0 * tc: c0 * tc + M].view(n, tc, 2 * kd)
            a = ext.attention_fwd(qkv.view(n, tc, -1)[:, :, :qd], kv[:, :, :kd], kv[:, :, kd:], self.heads,
                                  self.kv_heads, cfg.head_dim, None, None, None, None, valid,
                                  1.0 / math.sqrt(cfg.head_dim))[0]
            x = self._row_parallel(a.view(M, qd), lw.o, x)
            x = self._mlp(lw, x)

    # -- prefill / decode ---------------------------------------------------------------
    def set_namespace(self, start: torch.Tensor, end: torch.Tensor) -> None:
        """Row b may read chunks ``[start[b], end[b])`` of the memory."""
        self.namespace = (start.to(self.device, torch.int32).contiguous(), end.to(self.device, torch.int32).contiguous())
        self.page_table = None

    def set_page_table(self, table: torch.Tensor, counts: torch.Tensor) -> None:
        """Row b may read chunks ``table[b, :counts[b]]`` (a paged chunk cache's pages)."""
        n = counts.to(self.device, torch.int32).contiguous()
        self.namespace = (torch.zeros_like(n), n)
        self.page_table = table.to(self.device, torch.int32).contiguous()

    @torch.no_grad()
    @traced("pra.llama.prefill")
    def prefill(self, ids: torch.Tensor, lengths: torch.Tensor, max_new_tokens: int,
                row_batch: int | None = None, position_offset: torch.Tensor | None = None) -> torch.Tensor:
        """Left-aligned prompts ``ids`` ``[B, T]`` with ``lengths``: fills the local caches and
        returns the logits of each row's last prompt token ``[B, V]``.  ``row_batch`` bounds
        how many rows run through the layers at once (activation memory)."""
        cfg = self.cfg
        B, T = ids.shape
        ids = ids.to(self.device)
        lengths = lengths.to(self.device, torch.int32)
        max_len = T + max_new_tokens
        L = cfg.num_hidden_layers
        self.cache = torch.zeros((L, 2, B, max_len, self.kv_dim), device=self.device, dtype=torch.bfloat16)
        self.cache_len = lengths.clone()
        self.max_len = max_len
        # rotary position of cache slot t of row b: offset[b] + t (a long prompt's direct
        # tail continues the positions of its implicit head when they are natively legal)
        self.pos_offset = (position_offset.to(self.device, torch.int32).contiguous() if position_offset is not None
                           else torch.zeros(B, device=self.device, dtype=torch.int32))
        self._max_pos = int(self.pos_offset.max()) + max_len if B else max_len
        step = row_batch or B
        outs = [self._prefill_rows(ids[r: r + step], lengths[r: r + step], r) for r in range(0, B, step)]
        return torch.cat(outs)

    def _prefill_rows(self, ids, lengths, r0: int) -> torch.Tensor:
        cfg, ext = self.cfg, self.ext
        B, T = ids.shape
        max_len = self.max_len
        qd, kd = self.q_dim, self.kv_dim
        cos, sin = self.rope_tables(self._max_pos)
        M = B * T
        pos = (torch.arange(T, device=self.device, dtype=torch.int32)[None]
               + self.pos_offset[r0: r0 + B, None]).reshape(-1)
        rows = ((torch.arange(B, device=self.device, dtype=torch.int32)[:, None] + r0) * max_len
                + torch.arange(T, device=self.device, dtype=torch.int32)[None]).reshape(-1)
        valid = (torch.arange(T, device=self.device)[None] < lengths[:, None]).to(torch.uint8).contiguous()
        last = (torch.arange(B, device=self.device) * T + lengths.long() - 1)
        x = self._embed(ids)
        use_memory = self.memory is not None and self.namespace is not None and cfg.top_k_chunks > 0
        namespace = None
        if use_memory:
            namespace = (self.namespace[0][r0: r0 + B].contiguous(), self.namespace[1][r0: r0 + B].contiguous())
            self._row0 = r0
        for li, lw in enumerate(self.w.layers):
            h = self._norm(x, self._ln(lw.ln_in))
            qkv = self._gemm(h, lw.qkv, lw.qkv_bias)
            mem_args = (None, None, None, None)
            if use_memory and cfg.is_pra_layer(li):
                mem_idx, mem_len = self._route(li, qkv[last, :qd], B, namespace)
                mem_args = (self.memory.k(li), self.memory.v(li), mem_idx, mem_len)
            kc = self.cache[li, 0].view(-1, kd)
            vc = self.cache[li, 1].view(-1, kd)
            ext.rope_copy(qkv[:, qd: qd + kd], kc, rows, pos, cos, sin, self.kv_heads, cfg.head_dim)
            ext.rope_copy(qkv[:, qd + kd:], vc, rows, None, None, None, self.kv_heads, cfg.head_dim)
            ext.rope_copy(qkv[:, :qd], qkv[:, :qd], None, pos, cos, sin, self.heads, cfg.head_dim)
            k_rows = self.cache[li, 0][r0: r0 + B, :T]
            v_rows = self.cache[li, 1][r0: r0 + B, :T]
            a = ext.attention_fwd(qkv.view(B, T, -1)[:, :, :qd], k_rows, v_rows, self.heads, self.kv_heads,
                                  cfg.head_dim, *mem_args, valid, 1.0 / math.sqrt(cfg.head_dim))[0]
            x = self._row_parallel(a.view(M, qd), lw.o, x)
            x = self._mlp(lw, x)
        return self._logits(x[last])

    def _local_logits(self, x_last: torch.Tensor) -> torch.Tensor:
        """This rank's vocabulary slice of the logits ``[B, vocab_end - vocab_start]``."""
        h = self._norm(x_last.contiguous(), self.w.norm)
        return self._gemm(h, self.head_local)

    def _logits(self, x_last: torch.Tensor) -> torch.Tensor:
        """Full logits ``[B, V]`` (the slices of every rank gathered under tensor parallelism)."""
        local = self._local_logits(x_last)
        if self.tp is None:
            return local
        import torch.distributed as dist

        width = -(-self.w.head.shape[0] // self.tp_size)
        width = -(-width // 8) * 8
        padded = torch.zeros((local.shape[0], width), device=local.device, dtype=local.dtype)
        padded[:, : local.shape[1]] = local
        parts = [torch.empty_like(padded) for _ in range(self.tp_size)]
        dist.all_gather(parts, padded, group=self.tp.group)
        return torch.cat(parts, dim=1)[:, : self.w.head.shape[0]]

    def _greedy(self, x_last: torch.Tensor) -> torch.Tensor:
        """Greedy next token ids ``[B]``: each rank's (max, index) over its vocabulary slice, merged
        across ranks (ties go to the lowest index, as ``argmax`` over the full logits does)."""
        local = self._local_logits(x_last)
        best, idx = local.float().max(dim=-1)
        if self.tp is None:
            return idx
        pair = torch.stack([best, (idx + self.vocab_start).float()], dim=1)  # ids < 2^24 are exact in fp32
        every = self.tp.gather_small(pair).view(-1, self.tp_size, 2)
        score, ids = every[..., 0], every[..., 1]
        top = score.max(dim=1, keepdim=True).values
        return torch.where(score == top, ids, torch.full_like(ids, float("inf"))).min(dim=1).values.long()

    @torch.no_grad()
    @traced("pra.llama.decode_step")
    def decode_step(self, token_ids: torch.Tensor, sample: bool = False) -> torch.Tensor:
        """One token per row at position ``cache_len[b]``; returns logits ``[B, V]``, or with
        ``sample=True`` the greedy next token ids ``[B]`` (no full-vocabulary logits are formed
        under tensor parallelism)."""
        cfg, ext = self.cfg, self.ext
        B = token_ids.shape[0]
        qd, kd = self.q_dim, self.kv_dim
        cos, sin = self.rope_tables(self._max_pos)
        # one launch: embeddings, rotary positions, cache rows and new lengths of this step
        # folded RMSNorms: buffer 0 holds the per-tile row sums of squares of each layer's input
        # (from the prologue, then from the previous down projection), buffer 1 those of the
        # attention block's output (from the O projection)
        folded = getattr(self.w, "norm_folded", False) and self._decode_rows(token_ids.reshape(-1, 1))
        if folded and (self._ss is None or self._ss.device != self.device):
            self._ss = torch.zeros((2, self._ss_tiles, 64), device=self.device, dtype=torch.float32)
        x, pos, rows, new_len = ext.decode_prologue(token_ids.to(self.device, torch.long).reshape(-1).contiguous(),
                                                    self.cache_len, self.pos_offset, self.w.embed, self.max_len,
                                                    ss_out=self._ss[0] if folded else None)
        use_memory = self.memory is not None and self.namespace is not None and cfg.top_k_chunks > 0
        max_keys = cfg.memory_tokens_per_row + self.max_len
        for li, lw in enumerate(self.w.layers):
            h = x if folded else self._norm(x, self._ln(lw.ln_in))
            kc = self.cache[li, 0].view(B * self.max_len, kd)
            vc = self.cache[li, 1].view(B * self.max_len, kd)
            q = torch.empty((B, qd), device=self.device, dtype=torch.bfloat16)
            rq = qkv = None
            if self._decode_rows(h):
                # one GEMM: (folded input norm,) rotated q, rotated k and v straight into their
                # cache rows, routing query
                rq = torch.empty((B, self.route_dim), device=self.device, dtype=torch.bfloat16)
                norm = dict(ss_in=self._ss[0], ss_tiles=1 if li == 0 else self._ss_tiles, ss_dim=cfg.hidden_size,
                            ss_eps=cfg.rms_norm_eps) if folded else {}
                ext.decode_qkv_rope(h, lw.qkv_route, lw.qkv_route_bias, q, kc, vc, rows, pos, cos, sin, cfg.head_dim,
                                    qd, qd + kd, qd + 2 * kd, rq, **norm)
            else:
                qkv = self._gemm(h, lw.qkv, lw.qkv_bias)
                ext.rope_copy(qkv[:, qd: qd + kd], kc, rows, pos, cos, sin, self.kv_heads, cfg.head_dim)
                ext.rope_copy(qkv[:, qd + kd:], vc, rows, None, None, None, self.kv_heads, cfg.head_dim)
                ext.rope_copy(qkv[:, :qd], q, None, pos, cos, sin, self.heads, cfg.head_dim)
            mem_args = (None, None, None, None)
            routed = use_memory and cfg.is_pra_layer(li)
            if routed and self.overlap_routing:
                a = self._attend_overlapped(li, q, None if qkv is None else qkv[:, :qd], rq, new_len, max_keys)
            else:
                if routed:
                    mem_idx, mem_len = self._route(li, None if qkv is None else qkv[:, :qd], B, route_query=rq)
                    mem_args = (self.memory.k(li), self.memory.v(li), mem_idx, mem_len)
                a = ext.decode_attention(q, self.heads, self.kv_heads, cfg.head_dim, *mem_args, self.cache[li, 0],
                                         self.cache[li, 1], new_len, max_keys, self._split_for(B, max_keys), False)[0]
            if folded:
                x = self._row_parallel(a, lw.o, x, ss_out=self._ss[1])
                x = self._mlp(lw, x, ss=(self._ss[1], self._ss[0]))
            else:
                x = self._row_parallel(a, lw.o, x)
                x = self._mlp(lw, x)
        self.cache_len.copy_(new_len)  # in place: a captured step replays on the same tensors
        return self._greedy(x) if sample else self._logits(x)

    def _partials(self, B: int, n_split: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Split partials ``(o [B, H, n, Dh], (max, sum) [B, H, n, 2])`` shared by the phases of
        one overlapped decode attention; kept across layers and steps (stream order separates
        their uses: the next layer's splits are enqueued after this layer's merge)."""
        key = (B, n_split)
        if self._parts is None or self._parts[0] != key:
            H, D = self.heads, self.cfg.head_dim
            self._parts = (key, torch.empty((B, H, n_split, D), device=self.device, dtype=torch.float32),
                           torch.empty((B, H, n_split, 2), device=self.device, dtype=torch.float32))
        return self._parts[1], self._parts[2]

    def _attend_overlapped(self, li: int, q: torch.Tensor, q_rows, rq, new_len: torch.Tensor,
                           max_keys: int) -> torch.Tensor:
        """Decode attention of a routed layer with routing off the critical path.

        The local-window splits need only the queries and the cache, so they are enqueued first
        on the current stream; a high-priority side stream then scores the gists, selects the
        chunks (with the cross-GPU exchange under tensor parallelism) and attends over the
        selected memory rows into splits ``[0, n_mem)`` of the same partials; the merge runs
        after both.  Same result as the single launch: the merge weighs every split by its own
        (max, sum), whatever the split layout."""
        cfg, ext = self.cfg, self.ext
        B = q.shape[0]
        sk = self._split_for(B, max_keys)
        # memory splits of at most 256 keys: many short CTAs that start as soon as routing ends
        # and slot in between the local splits' CTAs
        msk = min(sk, 256)
        n_mem = max(1, -(-cfg.memory_tokens_per_row // msk))
        n_loc = -(-self.max_len // sk)
        part_o, part_ml = self._partials(B, n_mem + n_loc)
        kc, vc = self.cache[li, 0], self.cache[li, 1]
        H, Hkv, D = self.heads, self.kv_heads, cfg.head_dim
        common = dict(mem_splits=n_mem, mem_split_keys=msk, part_o=part_o, part_ml=part_ml)
        main = torch.cuda.current_stream(self.device)
        if self._route_stream is None:
            self._route_stream = torch.cuda.Stream(self.device, priority=-1)
        side = self._route_stream
        side.wait_stream(main)  # fork before the local splits: routing must not wait for them
        if self._local_ctas < 0:
            self._local_ctas = 2 * torch.cuda.get_device_properties(self.device).multi_processor_count
        ext.decode_attention(q, H, Hkv, D, None, None, None, None, kc, vc, new_len, 0, sk, False,
                             split_lo=n_mem, split_count=n_loc, phase=1, max_ctas=self._local_ctas, **common)
        with torch.cuda.stream(side):
            ext.set_launch_priority(True)  # also per kernel node when the step is captured
            try:
                mem_idx, mem_len = self._route(li, q_rows, B, route_query=rq)
                ext.decode_attention(q, H, Hkv, D, self.memory.k(li), self.memory.v(li), mem_idx, mem_len, kc, vc,
                                     new_len, 0, sk, False, split_lo=0, split_count=n_mem, phase=1, **common)
            finally:
                ext.set_launch_priority(False)
        main.wait_stream(side)
        return ext.decode_attention(q, H, Hkv, D, None, None, None, None, kc, vc, new_len, 0, sk, False, phase=2,
                                    **common)[0]

    # -- CUDA-graph decode ------------------------------------------------------------
    def capture_decode(self, sample: bool = False) -> None:
        """Capture one ``decode_step`` into a CUDA graph (after at least one eager step).

        Replays run the whole step (32 layers of GEMMs, routing, attention and the
        tensor-parallel collectives) as one graph launch; the collectives take their
        epochs from device counters, so replays stay in lockstep across ranks."""
        B = self.cache_len.shape[0]
        self._graph_ids = torch.zeros(B, dtype=torch.long, device=self.device)
        ar0 = self.tp.epoch_ar if self.tp is not None else 0
        ag0 = self.tp.epoch_ag if self.tp is not None else 0
        dg0 = self.tp.epoch_dg if self.tp is not None else 0
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        counter = _ext.launch_counter()
        was, before = counter.enabled, counter.launches
        counter.enabled = True  # count this library's kernels recorded in the graph
        with torch.cuda.graph(graph):
            self._graph_out = self.decode_step(self._graph_ids, sample=sample)
        self.graph_launches = counter.launches - before
        counter.launches, counter.enabled = before, was
        if self.tp is not None and ((self.tp.epoch_ar - ar0) % 2 or (self.tp.epoch_ag - ag0) % 2
                                    or (self.tp.epoch_dg - dg0) % 2):
            raise RuntimeError("a captured step must use both halves of each double buffer equally often")
        self._graph = graph

    def decode_step_graphed(self, token_ids: torch.Tensor) -> torch.Tensor:
        """``decode_step`` through the captured graph (returns the graph's static output: logits, or
        next token ids when captured with ``sample=True``)."""
        self._graph_ids.copy_(token_ids, non_blocking=True)
        self._graph.replay()
        return self._graph_out

    def release_graph(self) -> None:
        self._graph = None
        self._graph_out = None

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, lengths: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
        """Greedy decoding: ``[B, max_new_tokens]`` new token ids."""
        logits = self.prefill(ids, lengths, max_new_tokens)
        out = []
        tok = logits.float().argmax(-1)
        for _ in range(max_new_tokens):
            out.append(tok)
            if len(out) == max_new_tokens:
                break
            tok = self.decode_step(tok, sample=True)
        return torch.stack(out, dim=1)
