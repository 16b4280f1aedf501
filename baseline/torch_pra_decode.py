"""PRA decode on a Llama-family model in plain PyTorch + cuBLAS + NCCL (the comparison arm).

The reference implementation has no Llama-family model, no tensor parallelism and no
decode path for 8B models, so the decode benchmark compares against this module: the
reference's PRA decode semantics written the way a PyTorch user would, with no kernel,
model or engine of the framework being measured (it imports nothing from it).

Semantics (the reference's native-K/V PRA, restated for RoPE and GQA):
* memory build: every 64-token chunk is encoded as its own sequence (positions from 0);
  each layer keeps the chunk's post-RoPE K/V and one mean gist of its pre-RoPE keys over
  all KV heads (``src/pra_torch/gists/single.py`` mean gist, L2-normalised as in
  ``src/pra_torch/memory.py:504``);
* routing per layer and row: the pre-RoPE query of the current token averaged over each
  KV group (full KV width after an all-gather), cosine scores ``normalize(q) @ gists``
  (``src/pra_torch/memory.py:546-550``) and ``torch.topk`` of the chunks
  (``src/pra_torch/memory.py:656-675``); the selected chunks' K/V are gathered and
  attended together with the local cache under one softmax
  (``src/pra_torch/memory_batching.py:216-307``);
* tensor parallelism (Megatron layout): QKV and gate/up split by output columns, O and
  down by input rows with an NCCL all-reduce of their partial outputs; each rank keeps
  its KV heads of every chunk, the routing-query slices are all-gathered with NCCL.

Long prompts (``run_long_prompt``): the reference's prompt overflow
(``src/pra_torch/prompt.py:125-231``): each row's tokens before its last
``direct_window`` become 64-token chunks of its implicit ``#__head`` reference,
which only that row routes over (a per-row namespace of chunk ids); the direct
tail continues the head's positions when head + tail fit the native positions,
otherwise it restarts at 0 (``historical`` mode, ``src/pra_torch/config.py:194-202``).
"""

from __future__ import annotations

import math
import statistics
import time

import torch
import torch.distributed as dist
import torch.nn.functional as F

LLAMA3_8B = dict(hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336, layers=32, vocab=128256,
                 rope_theta=500000.0, eps=1e-5)
MISTRAL_7B = dict(hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336, layers=32, vocab=32768,
                  rope_theta=1000000.0, eps=1e-5, max_positions=32768)


class TorchPRALlama:
    def __init__(self, arch: dict, device, rank: int = 0, world: int = 1, seed: int = 0, std: float = 0.02,
                 top_k: int = 16, chunk_tokens: int = 64):
        self.a, self.device, self.rank, self.world = arch, torch.device(device), rank, world
        self.top_k, self.chunk_tokens = top_k, chunk_tokens
        d, dh = arch["hidden"], arch["head_dim"]
        self.h, self.hk = arch["heads"] // world, arch["kv_heads"] // world
        self.ns = None            # optional (start, end) [B]: row b routes over chunks [start, end)
        self.pos_offset = None    # optional [B] position of each row's first direct token
        self.qd, self.kd, self.f = self.h * dh, self.hk * dh, arch["inter"] // world
        gen = torch.Generator(device=self.device).manual_seed(seed + 1000 * rank)

        def rand(*shape):
            return (torch.randn(*shape, generator=gen, device=self.device) * std).to(torch.bfloat16)

        self.layers = [dict(ln1=torch.ones(d, device=self.device, dtype=torch.bfloat16),
                            qkv=rand(self.qd + 2 * self.kd, d), o=rand(d, self.qd),
                            ln2=torch.ones(d, device=self.device, dtype=torch.bfloat16),
                            gate_up=rand(2 * self.f, d), down=rand(d, self.f)) for _ in range(arch["layers"])]
        shared = torch.Generator(device=self.device).manual_seed(seed)
        self.embed = (torch.randn(arch["vocab"], d, generator=shared, device=self.device) * std).to(torch.bfloat16)
        self.head = (torch.randn(arch["vocab"], d, generator=shared, device=self.device) * std).to(torch.bfloat16)
        self.norm = torch.ones(d, device=self.device, dtype=torch.bfloat16)
        half = dh // 2
        self.inv_freq = 1.0 / (arch["rope_theta"] ** (torch.arange(0, half, device=self.device, dtype=torch.float64) / half))

    # -- building blocks ------------------------------------------------------------------
    def _rms(self, x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.a["eps"]) * w.float()).to(torch.bfloat16)

    def _rope(self, x, pos):
        """x [..., T, heads, dh] rotated at integer positions pos [..., T] (rotate-half form)."""
        ang = pos.double()[..., None] * self.inv_freq
        cos, sin = ang.cos().float()[..., None, :], ang.sin().float()[..., None, :]
        x1, x2 = x.float().chunk(2, dim=-1)
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(torch.bfloat16)

    def _all_reduce(self, t):
        if self.world > 1:
            dist.all_reduce(t)
        return t

    def _all_gather_cols(self, t):
        if self.world == 1:
            return t
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t.contiguous())
        return torch.cat(parts, dim=-1)

    def _mlp(self, lw, x):
        gu = self._rms(x, lw["ln2"]) @ lw["gate_up"].t()
        gate, up = gu.split(self.f, dim=-1)
        return x + self._all_reduce((F.silu(gate.float()) * up.float()).to(torch.bfloat16) @ lw["down"].t())

    def _split_qkv(self, qkv):
        q, k, v = qkv.split([self.qd, self.kd, self.kd], dim=-1)
        dh = self.a["head_dim"]
        return (q.unflatten(-1, (self.h, dh)), k.unflatten(-1, (self.hk, dh)), v.unflatten(-1, (self.hk, dh)))

    # -- memory --------------------------------------------------------------------------
    @torch.no_grad()
    def build_memory(self, chunks: torch.Tensor, batch: int = 256) -> None:
        """chunks [C, Tc] token ids -> per-layer K/V pools [C*Tc, kd] and normalised gists [C, kv_total]."""
        C, Tc = chunks.shape
        L, dh = self.a["layers"], self.a["head_dim"]
        self.mem_k = torch.empty((L, C * Tc, self.kd), device=self.device, dtype=torch.bfloat16)
        self.mem_v = torch.empty_like(self.mem_k)
        gists = torch.empty((L, C, self.kd), device=self.device, dtype=torch.float32)
        pos = torch.arange(Tc, device=self.device)
        for c0 in range(0, C, batch):
            ids = chunks[c0: c0 + batch].to(self.device)
            n = ids.shape[0]
            x = self.embed[ids]
            for li, lw in enumerate(self.layers):
                q, k, v = self._split_qkv(self._rms(x, lw["ln1"]) @ lw["qkv"].t())
                gists[li, c0: c0 + n] = k.float().mean(dim=1).flatten(1)  # pre-RoPE key mean
                q, k = self._rope(q, pos), self._rope(k, pos)
                rows = slice(c0 * Tc, (c0 + n) * Tc)
                self.mem_k[li, rows] = k.flatten(2).reshape(n * Tc, self.kd)
                self.mem_v[li, rows] = v.flatten(2).reshape(n * Tc, self.kd)
                a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                   is_causal=True, enable_gqa=True)
                x = x + self._all_reduce(a.transpose(1, 2).flatten(2) @ lw["o"].t())
                x = self._mlp(lw, x)
        full = torch.stack([self._all_gather_cols(gists[li]) for li in range(L)])
        self.gists = F.normalize(full, dim=-1, eps=1e-12)  # [L, C, kv_total]
        self.n_chunks = C

    def _route(self, li, q_pre):
        """q_pre [B, h, dh] pre-RoPE queries -> selected chunk ids [B, top_k]."""
        g = self.h // self.hk
        rq = q_pre.float().unflatten(1, (self.hk, g)).mean(2).flatten(1)  # group mean [B, kd]
        rq = F.normalize(self._all_gather_cols(rq), dim=-1, eps=1e-12)
        scores = rq @ self.gists[li].t()
        if self.ns is not None:  # each row only sees its own namespace of chunks
            start, end = self.ns
            start, end = start[self._rows], end[self._rows]
            ids = torch.arange(scores.shape[1], device=self.device)
            scores = scores.masked_fill((ids < start[:, None]) | (ids >= end[:, None]), float("-inf"))
        return scores.topk(self.top_k, dim=-1).indices

    def _memory_kv(self, li, chunk_ids):
        """K/V rows of the selected chunks [B, top_k * Tc, hk, dh]."""
        Tc, dh = self.chunk_tokens, self.a["head_dim"]
        rows = (chunk_ids[..., None] * Tc + torch.arange(Tc, device=self.device)).flatten(1)
        return (self.mem_k[li][rows].unflatten(-1, (self.hk, dh)), self.mem_v[li][rows].unflatten(-1, (self.hk, dh)))

    # -- prompt and decode ----------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, prompts: torch.Tensor, max_new: int, row_batch: int = 4) -> torch.Tensor:
        """Causal prefill of [B, T] prompts with memory routed on each row's last token; returns next ids."""
        B, T = prompts.shape
        L, dh = self.a["layers"], self.a["head_dim"]
        self.max_len = T + max_new
        self.cache_k = torch.zeros((L, B, self.max_len, self.hk, dh), device=self.device, dtype=torch.bfloat16)
        self.cache_v = torch.zeros_like(self.cache_k)
        self.length = T
        out = []
        offset = self.pos_offset if self.pos_offset is not None else torch.zeros(B, dtype=torch.long,
                                                                                   device=self.device)
        for r0 in range(0, B, row_batch):
            ids = prompts[r0: r0 + row_batch].to(self.device)
            n = ids.shape[0]
            self._rows = torch.arange(r0, r0 + n, device=self.device)
            pos = offset[r0: r0 + n, None] + torch.arange(T, device=self.device)[None]
            x = self.embed[ids]
            for li, lw in enumerate(self.layers):
                q, k, v = self._split_qkv(self._rms(x, lw["ln1"]) @ lw["qkv"].t())
                mk, mv = self._memory_kv(li, self._route(li, q[:, -1]))
                q, k = self._rope(q, pos), self._rope(k, pos)
                self.cache_k[li, r0: r0 + n, :T], self.cache_v[li, r0: r0 + n, :T] = k, v
                keys, vals = torch.cat([mk, k], dim=1), torch.cat([mv, v], dim=1)
                M = mk.shape[1]
                mask = torch.ones((T, M + T), device=self.device, dtype=torch.bool)
                mask[:, M:] = torch.ones((T, T), device=self.device, dtype=torch.bool).tril()
                a = F.scaled_dot_product_attention(q.transpose(1, 2), keys.transpose(1, 2), vals.transpose(1, 2),
                                                   attn_mask=mask, enable_gqa=True)
                x = x + self._all_reduce(a.transpose(1, 2).flatten(2) @ lw["o"].t())
                x = self._mlp(lw, x)
            out.append(self._greedy(x[:, -1]))
        return torch.cat(out)

    def _greedy(self, x_last):
        return (self._rms(x_last, self.norm) @ self.head.t()).float().argmax(-1)

    @torch.no_grad()
    def decode_step(self, tok: torch.Tensor) -> torch.Tensor:
        """One token per row (all rows at the same length); returns the greedy next ids."""
        t = self.length
        x = self.embed[tok][:, None]
        B = tok.shape[0]
        self._rows = torch.arange(B, device=self.device)
        offset = self.pos_offset if self.pos_offset is not None else torch.zeros(B, dtype=torch.long,
                                                                                   device=self.device)
        pos = (offset + t)[:, None]
        for li, lw in enumerate(self.layers):
            q, k, v = self._split_qkv(self._rms(x, lw["ln1"]) @ lw["qkv"].t())
            mk, mv = self._memory_kv(li, self._route(li, q[:, 0]))
            q, k = self._rope(q, pos), self._rope(k, pos)
            self.cache_k[li, :, t], self.cache_v[li, :, t] = k[:, 0], v[:, 0]
            keys = torch.cat([mk, self.cache_k[li, :, : t + 1]], dim=1)
            vals = torch.cat([mv, self.cache_v[li, :, : t + 1]], dim=1)
            a = F.scaled_dot_product_attention(q.transpose(1, 2), keys.transpose(1, 2), vals.transpose(1, 2),
                                               enable_gqa=True)
            x = x + self._all_reduce(a.transpose(1, 2).flatten(2) @ lw["o"].t())
            x = self._mlp(lw, x)
        self.length = t + 1
        return self._greedy(x[:, 0])


def run(*, batch: int = 64, prompt_tokens: int = 4096, memory_tokens: int = 1 << 20, top_k: int = 16,
        steps: int = 16, warmup: int = 3, seed: int = 0, arch: dict | None = None) -> dict:
    """Memory build, prefill and timed greedy decode steps (max over ranks); same workload as the
    framework's decode benchmark, with every step's ids copied in from pinned memory and read back."""
    arch = arch or LLAMA3_8B
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    device = torch.device("cuda", torch.cuda.current_device())
    model = TorchPRALlama(arch, device, rank, world, seed=seed, top_k=top_k)
    gen = torch.Generator().manual_seed(seed + 1)
    chunks = torch.randint(0, arch["vocab"], (memory_tokens // 64, 64), generator=gen)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    model.build_memory(chunks)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    prompts = torch.randint(0, arch["vocab"], (batch, prompt_tokens), generator=gen)
    t0 = time.perf_counter()
    tok = model.prefill(prompts, warmup + steps + 1)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    host_in = torch.empty(batch, dtype=torch.int64).pin_memory()
    host_out = torch.empty(batch, dtype=torch.int64).pin_memory()
    host_in.copy_(tok.cpu())
    for _ in range(warmup):
        host_out.copy_(model.decode_step(host_in.to(device, non_blocking=True)), non_blocking=True)
        torch.cuda.synchronize()
        host_in.copy_(host_out)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    per_step = []
    wall0 = time.perf_counter()
    for _ in range(steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        host_out.copy_(model.decode_step(host_in.to(device, non_blocking=True)), non_blocking=True)
        e.record()
        torch.cuda.current_stream().synchronize()
        host_in.copy_(host_out)
        per_step.append(s.elapsed_time(e))
    wall = time.perf_counter() - wall0

    def worst(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    per_step = sorted(worst(v) for v in per_step)
    device_s = worst(sum(per_step) / 1000.0)
    return {"tokens_per_s": batch * steps / device_s, "e2e_tokens_per_s": batch * steps / worst(wall),
            "tpot_p50_ms": statistics.median(per_step), "tpot_p90_ms": per_step[min(len(per_step) - 1,
                                                                                     int(0.9 * len(per_step)))],
            "build_tokens_per_s": memory_tokens / worst(build_s),
            "prefill_tokens_per_s": batch * prompt_tokens / worst(prefill_s), "memory_tokens": memory_tokens,
            "tp": world, "batch": batch, "prompt_tokens": prompt_tokens, "top_k_chunks": top_k,
            "h2d_bytes_per_step": batch * 8, "d2h_bytes_per_step": batch * 8}


def run_long_prompt(*, batch: int = 16, prompt_tokens: int = 131072, direct_window: int = 4096, top_k: int = 16,
                    new_tokens: int = 256, seed: int = 0, arch: dict | None = None) -> dict:
    """The long-prompt workload: ``batch`` prompts of ``prompt_tokens`` uniform-random ids; each
    row's head (all but its last ``direct_window`` tokens) becomes its own 64-token chunks,
    then the tails are prefilled and ``new_tokens`` greedy tokens decoded (device time with
    CUDA events, max over ranks)."""
    arch = arch or MISTRAL_7B
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    device = torch.device("cuda", torch.cuda.current_device())
    model = TorchPRALlama(arch, device, rank, world, seed=seed, top_k=top_k)
    gen = torch.Generator().manual_seed(seed + 1)
    prompts = torch.randint(0, arch["vocab"], (batch, prompt_tokens), generator=gen)
    head_len = max(0, prompt_tokens - direct_window)
    if head_len % 64:
        raise ValueError("this arm expects heads that are whole 64-token chunks")
    per_row = head_len // 64
    chunks = prompts[:, :head_len].reshape(batch * per_row, 64)
    legal = head_len + direct_window <= arch.get("max_positions", 1 << 30)
    model.ns = (torch.arange(batch, device=device) * per_row, (torch.arange(batch, device=device) + 1) * per_row)
    model.pos_offset = torch.full((batch,), head_len if legal else 0, dtype=torch.long, device=device)

    def timed(fn):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = fn()
        e.record()
        torch.cuda.synchronize()
        return out, s.elapsed_time(e)

    _, build_ms = timed(lambda: model.build_memory(chunks))
    tok, prefill_ms = timed(lambda: model.prefill(prompts[:, head_len:], new_tokens + 1))
    per_step = []
    for _ in range(new_tokens - 1):
        tok, ms = timed(lambda: model.decode_step(tok))
        per_step.append(ms)

    def worst(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    per_step = [worst(v) for v in per_step]
    build_ms, prefill_ms = worst(build_ms), worst(prefill_ms)
    return {"decode_tokens_per_s": batch * len(per_step) / (sum(per_step) / 1000),
            "tpot_p50_ms": statistics.median(per_step),
            "prefill_tokens_per_s": batch * prompt_tokens / ((build_ms + prefill_ms) / 1000),
            "head_build_tokens_per_s": batch * head_len / (build_ms / 1000),
            "tail_prefill_tokens_per_s": batch * direct_window / (prefill_ms / 1000), "head_tokens": batch * head_len,
            "batch": batch, "prompt_tokens": prompt_tokens, "direct_window": direct_window,
            "new_tokens": new_tokens, "decode_steps": len(per_step), "tp": world,
            "position_offset": int(model.pos_offset[0])}
