"""Decode benchmark of a PRA Llama-family model with a large chunk memory.

Workload (synthetic, random-init weights): ``batch`` requests, each with a
``prompt_tokens`` direct window of uniform-random token ids, all reading one shared
memory of ``refs`` references of ``ref_tokens`` uniform-random tokens each, cut into
``chunk_tokens`` chunks with one mean gist per chunk; ``top_k_chunks`` chunks are
routed per layer and step.  After the memory build and the prefill, ``warmup``
untimed and ``steps`` timed greedy decode steps run through the engine's public
``decode_step``; every step copies its input token ids host->device from pinned
memory and reads the sampled ids back (the end-to-end loop a server runs).

Reported: decode tokens/s over the timed steps (device time, max over ranks) and the
p50 / p90 time per output token from per-step CUDA events.
"""

from __future__ import annotations

import statistics
import time

import torch

from ..models.llama import PRESETS
from .llama_engine import LlamaWeights, PRALlamaEngine


def run_decode_benchmark(*, model: str = "llama3-8b", batch: int = 64, prompt_tokens: int = 4096, refs: int = 32,
                         ref_tokens: int = 32768, chunk_tokens: int = 64, top_k_chunks: int = 16, steps: int = 16,
                         warmup: int = 3, tp=None, seed: int = 0, prefill_rows: int = 4,
                         build_chunks: int = 512, clocks=None, counter=None, graphs: bool = True) -> dict:
    rank = tp.rank if tp is not None else 0
    world = tp.world if tp is not None else 1
    device = torch.device("cuda", torch.cuda.current_device())
    cfg = PRESETS[model](chunk_tokens=chunk_tokens, top_k_chunks=top_k_chunks, direct_window=prompt_tokens)
    weights = LlamaWeights.random(cfg, device, seed=seed, tp_rank=rank, tp_size=world)
    engine = PRALlamaEngine(weights, device, tp=tp)
    gen = torch.Generator().manual_seed(seed + 1)
    n_chunks = refs * ref_tokens // chunk_tokens
    chunks = torch.randint(0, cfg.vocab_size, (n_chunks, chunk_tokens), generator=gen)
    lengths = torch.full((n_chunks,), chunk_tokens, dtype=torch.int32)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    engine.build_memory(chunks, lengths, batch_chunks=build_chunks)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    engine.set_namespace(torch.zeros(batch, dtype=torch.int32), torch.full((batch,), n_chunks, dtype=torch.int32))
    prompts = torch.randint(0, cfg.vocab_size, (batch, prompt_tokens), generator=gen)
    plen = torch.full((batch,), prompt_tokens, dtype=torch.int32)
    t0 = time.perf_counter()
    logits = engine.prefill(prompts, plen, warmup + steps + 1, row_batch=prefill_rows)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0

    host_tok = torch.empty(batch, dtype=torch.int64).pin_memory()
    host_out = torch.empty(batch, dtype=torch.int64).pin_memory()
    tok = logits.float().argmax(-1)
    host_tok.copy_(tok.cpu())

    step_fn = lambda ids: engine.decode_step(ids, sample=True)  # noqa: E731  greedy ids, vocabulary-parallel

    def one_step():
        ids = host_tok.to(device, non_blocking=True)
        nxt = step_fn(ids)
        host_out.copy_(nxt, non_blocking=True)
        return nxt

    for i in range(warmup):
        one_step()
        torch.cuda.synchronize()
        host_tok.copy_(host_out)
        if graphs and i == 0:  # capture after one eager step, replay for the rest
            engine.capture_decode(sample=True)
            step_fn = engine.decode_step_graphed
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    if tp is not None:
        tp.barrier()
    torch.cuda.synchronize()
    sampler = clocks if clocks is not None else None
    if sampler is not None:
        sampler.__enter__()
    if counter is not None:
        counter.reset()
        counter.enabled = True
    wall0 = time.perf_counter()
    for i in range(steps):
        events[i][0].record()
        one_step()
        events[i][1].record()
        torch.cuda.current_stream().synchronize()  # the sampled ids are read before the next step
        host_tok.copy_(host_out)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    launches = None
    if counter is not None:
        counter.enabled = False
        launches = engine.graph_launches * steps if graphs else counter.launches
    if sampler is not None:
        sampler.__exit__(None, None, None)
    if graphs:
        engine.release_graph()
    per_step = [a.elapsed_time(b) for a, b in events]
    device_s = sum(per_step) / 1000.0
    if tp is not None:
        device_s = tp.max_scalar(device_s)
        wall = tp.max_scalar(wall)
        per_step = [tp.max_scalar(x) for x in per_step]
    per_step.sort()
    memory_tokens = n_chunks * chunk_tokens
    return {
        "tokens_per_s": batch * steps / device_s,
        "e2e_tokens_per_s": batch * steps / wall,
        "tpot_p50_ms": statistics.median(per_step),
        "tpot_p90_ms": per_step[min(len(per_step) - 1, int(0.9 * len(per_step)))],
        "build_tokens_per_s": memory_tokens / build_s,
        "prefill_tokens_per_s": batch * prompt_tokens / prefill_s,
        "memory_tokens": memory_tokens,
        "model": model,
        "params_b": cfg.parameter_count() / 1e9,
        "batch": batch,
        "prompt_tokens": prompt_tokens,
        "top_k_chunks": top_k_chunks,
        "chunk_tokens": chunk_tokens,
        "tp": world,
        "h2d_bytes_per_step": batch * 8,
        "d2h_bytes_per_step": batch * 8,
        "memory_gb_per_gpu": engine.memory.nbytes() / 1e9,
        "gpu_launches": launches,
        "cuda_graphs": graphs,
    }
