"""Routing + memory-attention sweep of one PRA layer with a chunk-sharded memory.

Qwen2-7B PRA layer shapes (28 query heads over 4 KV heads, head_dim 128, routing in
the 512-wide key space), a decode batch of ``rows`` queries, and a chunk memory of
Gaussian random K/V sharded by chunk across the ranks of a group (rank r holds chunks
``[r * per, (r + 1) * per)`` with all KV heads).  Each of the ``G`` gists of a chunk is
the mean key of one of its ``64 / G`` -token slices.  One layer step:

1. each rank scores its chunks' gists on the tensor cores (bf16 normalised queries x
   bf16 normalised gists), takes a chunk's best gist, and keeps its exact fp32 top-k
   (radix select of candidates + fp32 rescoring);
2. the ranks' candidates are all-gathered over NVLink peer stores and merged into the
   global top-k (identical on every rank);
3. each rank computes the attention partial (max, sum, unnormalised output) of every
   query head over the selected chunks IT holds -- attention runs where the chunk
   lives, no K/V crosses NVLink;
4. the partials are all-gathered and combined into the output on every rank.

The baseline arm runs the same math with PyTorch operators (cuBLAS scores,
``torch.topk``, gathers, softmax attention) and NCCL all-gathers.  All timings are
CUDA events on the launching stream, max over ranks.
"""

from __future__ import annotations

import math
import statistics

import torch
import torch.nn.functional as F

from ..ops import _ext
from .routing import select_chunks

HEADS, KV_HEADS, HEAD_DIM = 28, 4, 128
KV_DIM = KV_HEADS * HEAD_DIM
CHUNK = 64


class ShardedLayerMemory:
    def __init__(self, total_tokens: int, gists_per_chunk: int, device, rank: int = 0, world: int = 1,
                 seed: int = 0):
        if CHUNK % gists_per_chunk:
            raise ValueError("gists per chunk must divide the chunk length")
        self.G = gists_per_chunk
        self.C = total_tokens // CHUNK
        per = ((self.C + world - 1) // world + 7) // 8 * 8
        self.c0 = min(self.C, rank * per)
        self.c1 = min(self.C, self.c0 + per)
        n = self.c1 - self.c0
        self.n = n
        dev = torch.device(device)
        gen = torch.Generator(device=dev).manual_seed(seed * 1000 + rank)
        self.pool = torch.empty((max(n, 1) * CHUNK, 2 * KV_DIM), device=dev, dtype=torch.bfloat16)
        block = 1 << 18
        for r0 in range(0, n * CHUNK, block):
            r1 = min(n * CHUNK, r0 + block)
            self.pool[r0:r1] = torch.randn((r1 - r0, 2 * KV_DIM), generator=gen, device=dev).to(torch.bfloat16)
        keys = self.pool[: n * CHUNK, :KV_DIM].float().view(n, self.G, CHUNK // self.G, KV_DIM)
        self.gn = F.normalize(keys.mean(2).reshape(n * self.G, KV_DIM), dim=-1, eps=1e-12).contiguous()
        if n == 0:
            self.gn = torch.zeros((self.G, KV_DIM), device=dev)
        self.gn_bf16 = self.gn.to(torch.bfloat16)
        ids = torch.arange(self.C, device=dev, dtype=torch.int32)
        self.chunk_len = torch.full((self.C,), CHUNK, device=dev, dtype=torch.int32)
        owned = (ids >= self.c0) & (ids < self.c1)
        self.chunk_row0 = torch.where(owned, (ids - self.c0) * CHUNK, torch.full_like(ids, -1))
        self.local_row0 = torch.arange(max(n, 1), device=dev, dtype=torch.int32) * CHUNK

    def nbytes(self) -> int:
        return self.pool.numel() * 2 + self.gn.numel() * 6


def fused_layer_step(mem: ShardedLayerMemory, rq: torch.Tensor, q: torch.Tensor, k: int, comm=None,
                     timers: dict | None = None) -> torch.Tensor:
    """Routing + memory attention of one layer with this library's kernels."""
    ext = _ext.require()
    rows = rq.shape[0]
    world = comm.world if comm is not None else 1

    def mark(name):
        if timers is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            timers.setdefault(name, []).append(e)

    mark("start")
    rqn = F.normalize(rq, dim=-1, eps=1e-12).to(torch.bfloat16)
    scores = torch.empty((rows, max(mem.n, 1) * mem.G), device=rq.device, dtype=torch.float32)
    ext.gemm("tn_f32", rqn, mem.gn_bf16, None, scores, None, None, 1.0, 0.0, None)
    zeros = torch.zeros(rows, device=rq.device, dtype=torch.int32)
    ends = torch.full((rows,), mem.n, device=rq.device, dtype=torch.int32)
    k_cand = min(max(4 * k, k), 512)
    mem_idx, mem_len, _ = select_chunks(ext, scores, rq, mem.gn, zeros, ends, mem.chunk_len, mem.local_row0, k,
                                        k_cand, -1, k * CHUNK, gists_per_chunk=mem.G, id_offset=mem.c0,
                                        comm=comm if world > 1 else None, global_len=mem.chunk_len,
                                        global_row0=mem.chunk_row0)
    mark("routed")
    pool_k, pool_v = mem.pool[:, :KV_DIM], mem.pool[:, KV_DIM:]
    res = ext.decode_attention(q, HEADS, KV_HEADS, HEAD_DIM, pool_k, pool_v, mem_idx, mem_len, None, None, None,
                               k * CHUNK, 512, world > 1)
    if world == 1:
        out = res[0]
    else:
        parts = torch.cat([res[1], res[2]], dim=-1).view(rows, HEADS * (HEAD_DIM + 2))
        gathered = comm.all_gather_columns(parts)
        out = ext.combine_partials(gathered, world, HEADS, HEAD_DIM)
    mark("done")
    return out


def baseline_layer_step(mem: ShardedLayerMemory, rq: torch.Tensor, q: torch.Tensor, k: int, group=None,
                        timers: dict | None = None) -> torch.Tensor:
    """The same layer step with PyTorch operators and NCCL (the baseline arm)."""
    import torch.distributed as dist

    world = dist.get_world_size(group) if group is not None else 1
    rows = rq.shape[0]

    def mark(name):
        if timers is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            timers.setdefault(name, []).append(e)

    mark("start")
    qn = F.normalize(rq, dim=-1, eps=1e-12)
    scores = (qn @ mem.gn.t()).view(rows, -1, mem.G).amax(-1)          # [B, n] fp32
    kk = min(k, max(mem.n, 1))
    top_s, top_i = torch.topk(scores, kk, dim=1)
    top_i = top_i + mem.c0
    if world > 1:
        s_all = [torch.empty_like(top_s) for _ in range(world)]
        i_all = [torch.empty_like(top_i) for _ in range(world)]
        dist.all_gather(s_all, top_s, group=group)
        dist.all_gather(i_all, top_i, group=group)
        cand_s, cand_i = torch.cat(s_all, 1), torch.cat(i_all, 1)
        best = torch.topk(cand_s, k, dim=1).indices
        sel = torch.gather(cand_i, 1, best)
    else:
        sel = top_i
    mark("routed")
    local = (sel >= mem.c0) & (sel < mem.c1)
    rows_idx = ((sel - mem.c0).clamp(0, max(mem.n - 1, 0))[..., None] * CHUNK
                + torch.arange(CHUNK, device=rq.device)).view(rows, -1)
    keys = mem.pool[rows_idx, :KV_DIM].float().view(rows, -1, KV_HEADS, HEAD_DIM)
    vals = mem.pool[rows_idx, KV_DIM:].float().view(rows, -1, KV_HEADS, HEAD_DIM)
    mask = local[..., None].expand(rows, sel.shape[1], CHUNK).reshape(rows, -1)
    g = HEADS // KV_HEADS
    qh = q.float().view(rows, KV_HEADS, g, HEAD_DIM)
    s = torch.einsum("bhgd,bkhd->bhgk", qh, keys) / math.sqrt(HEAD_DIM)
    s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
    m = s.amax(-1, keepdim=True)
    p = torch.exp(s - m.clamp_min(-1e30)).nan_to_num(0.0)
    o = torch.einsum("bhgk,bkhd->bhgd", p, vals).reshape(rows, HEADS, HEAD_DIM)
    l_sum = p.sum(-1).reshape(rows, HEADS)
    m = m.reshape(rows, HEADS)
    if world > 1:
        parts = torch.cat([o, m[..., None], l_sum[..., None]], -1)
        gathered = [torch.empty_like(parts) for _ in range(world)]
        dist.all_gather(gathered, parts, group=group)
        allp = torch.stack(gathered)                                   # [W, B, H, D + 2]
        mm = allp[..., HEAD_DIM].amax(0)
        w = torch.exp(allp[..., HEAD_DIM] - mm).nan_to_num(0.0)
        num = (allp[..., :HEAD_DIM] * w[..., None]).sum(0)
        den = (allp[..., HEAD_DIM + 1] * w).sum(0)
        out = (num / den.clamp_min(1e-30)[..., None]).reshape(rows, -1).to(torch.bfloat16)
    else:
        out = (o / l_sum.clamp_min(1e-30)[..., None]).reshape(rows, -1).to(torch.bfloat16)
    mark("done")
    return out


def run_sweep(memory_tokens=(1 << 16, 1 << 20, 1 << 24), gists=(1, 4), top_k=(4, 16, 64), rows: int = 64,
              iters: int = 20, warmup: int = 3, comm=None, group=None, arms=("fused", "baseline"), seed: int = 0):
    """Yields one result dict per (memory, G, k, arm): route / attention / total microseconds
    (median over iterations, max over ranks) and the achieved HBM bandwidth of the
    attention's K/V reads on this rank."""
    rank = comm.rank if comm is not None else 0
    world = comm.world if comm is not None else 1
    dev = torch.device("cuda", torch.cuda.current_device())
    for tokens in memory_tokens:
        for G in gists:
            mem = ShardedLayerMemory(tokens, G, dev, rank, world, seed)
            gen = torch.Generator(device=dev).manual_seed(seed + 7)
            rq = torch.randn((rows, KV_DIM), generator=gen, device=dev)
            q = torch.randn((rows, HEADS * HEAD_DIM), generator=gen, device=dev).to(torch.bfloat16)
            for k in top_k:
                for arm in arms:
                    step = fused_layer_step if arm == "fused" else baseline_layer_step
                    extra = {"comm": comm} if arm == "fused" else {"group": group}
                    for _ in range(warmup):
                        step(mem, rq, q, k, **extra)
                    torch.cuda.synchronize()
                    if comm is not None:
                        comm.barrier()
                    timers: dict = {}
                    for _ in range(iters):
                        step(mem, rq, q, k, timers=timers, **extra)
                    torch.cuda.synchronize()
                    route = [a.elapsed_time(b) * 1000 for a, b in zip(timers["start"], timers["routed"])]
                    attn = [a.elapsed_time(b) * 1000 for a, b in zip(timers["routed"], timers["done"])]
                    total = [a.elapsed_time(b) * 1000 for a, b in zip(timers["start"], timers["done"])]
                    med = [statistics.median(x) for x in (route, attn, total)]
                    if comm is not None:
                        med = [comm.max_scalar(x) for x in med]
                    local_bytes = rows * k * CHUNK * 2 * KV_DIM * 2 / world
                    yield {"memory_tokens": tokens, "gists_per_chunk": G, "chunk_top_k": k, "arm": arm,
                           "n_gpus": world, "rows": rows, "route_us": med[0], "attention_us": med[1],
                           "total_us": med[2], "attention_kv_gbs": local_bytes / (med[1] * 1e-6) / 1e9,
                           "memory_gb_per_gpu": mem.nbytes() / 1e9}
            del mem
            torch.cuda.empty_cache()
