"""Small, fixed workloads for kernel profiling (``ncu``) and per-step kernel tables.

Every case runs a few warm-up steps and exits 0, so it can run first without a
profiler and then under ``ncu`` on one GPU with the same arguments::

    python -m pdattention_b200.profiling train-small       # TinyGPT-PRA steps, 2 rows
    python -m pdattention_b200.profiling decode-small      # Llama-3-8B decode, 512 memory chunks
    python -m pdattention_b200.profiling train-table       # torch.profiler kernel table of one step (8 rows)
    python -m pdattention_b200.profiling decode-table      # kernel table of one decode step (64 rows)
    python -m pdattention_b200.profiling attention-fwd     # forward attention kernels, tcgen05 vs mma.sync
    torchrun --nproc-per-node N -m pdattention_b200.profiling decode-table-tp   # TP decode step table

The ``*-small`` cases keep device memory to a few GB so full ``ncu`` captures of one
launch end quickly.  Numbers printed under a profiler are not benchmark values.
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
import time
from pathlib import Path

import torch


def _train_step_fn(rows: int):
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    import bench  # the benchmark's data and model set-up

    bench.PER_GPU_BATCH = rows
    from pdattention_b200.data import WordIdTokenizer

    tmp = Path(tempfile.mkdtemp())
    tok = WordIdTokenizer(bench.VOCAB)
    bench._make_data(tmp, max(16, 4 * rows), 0, tok)
    step, _, counter = bench._pra_arm(tmp, tok, 0, 1)
    return step, counter


def train_small(steps: int = 3) -> None:
    step, _ = _train_step_fn(2)
    batches = step.batches(steps)
    for b in batches:
        step(b)
    torch.cuda.synchronize()
    print("ok")


def _decode_engine(memory_chunks: int, prompt: int, rows: int):
    from .inference.llama_engine import LlamaWeights, PRALlamaEngine
    from .models.llama import PRESETS

    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = PRESETS["llama3-8b"](chunk_tokens=64, top_k_chunks=16, direct_window=prompt)
    engine = PRALlamaEngine(LlamaWeights.random(cfg, dev), dev)
    gen = torch.Generator().manual_seed(0)
    engine.build_memory(torch.randint(0, cfg.vocab_size, (memory_chunks, 64), generator=gen),
                        torch.full((memory_chunks,), 64, dtype=torch.int32))
    engine.set_namespace(torch.zeros(rows, dtype=torch.int32), torch.full((rows,), memory_chunks, dtype=torch.int32))
    logits = engine.prefill(torch.randint(0, cfg.vocab_size, (rows, prompt), generator=gen),
                            torch.full((rows,), prompt, dtype=torch.int32), 16, row_batch=8)
    return engine, logits.float().argmax(-1)


def decode_small(steps: int = 3) -> None:
    engine, tok = _decode_engine(512, 2048, 64)
    for _ in range(steps):
        tok = engine.decode_step(tok).float().argmax(-1)
    torch.cuda.synchronize()
    print("ok")


def _table(fn, rows: int = 30, host_rows: int = 0) -> None:
    """Kernel table (by CUDA time) of ``fn``; with ``host_rows`` also the host-side table (by
    self CPU time: Python-level ops, launches and copies issued by the host)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    averages = prof.key_averages()
    print(averages.table(sort_by="cuda_time_total", row_limit=rows, max_name_column_width=70))
    if host_rows:
        print(averages.table(sort_by="self_cpu_time_total", row_limit=host_rows, max_name_column_width=70))


def train_table() -> None:
    step, counter = _train_step_fn(8)
    batches = step.batches(6)
    for b in batches[:4]:
        step(b)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    step(batches[4])
    torch.cuda.synchronize()
    print(f"step wall ms {1000 * (time.perf_counter() - t0):.2f}")
    _table(lambda: step(batches[5]), host_rows=25)


def decode_table() -> None:
    engine, tok = _decode_engine(1024, 4096, 64)
    for _ in range(3):
        tok = engine.decode_step(tok).float().argmax(-1)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(5):
        tok = engine.decode_step(tok).float().argmax(-1)
    torch.cuda.synchronize()
    print(f"step wall ms {1000 * (time.perf_counter() - t0) / 5:.2f}")
    _table(lambda: engine.decode_step(tok))


def decode_table_tp(memory_chunks: int = 16384) -> None:
    """Kernel table of one graph-replayed decode step on rank 0 of a tensor-parallel group
    (run under ``torch.distributed.run``; 64 rows, 4096-token prompts, 1M-token memory)."""
    import datetime
    import os

    import torch.distributed as dist

    from .inference.llama_engine import LlamaWeights, PRALlamaEngine
    from .models.llama import PRESETS
    from .parallel.tp import TensorParallel

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    tp = TensorParallel()
    dev = torch.device("cuda", local)
    cfg = PRESETS["llama3-8b"](chunk_tokens=64, top_k_chunks=16, direct_window=4096)
    engine = PRALlamaEngine(LlamaWeights.random(cfg, dev, tp_rank=tp.rank, tp_size=tp.world), dev, tp=tp)
    gen = torch.Generator().manual_seed(0)
    engine.build_memory(torch.randint(0, cfg.vocab_size, (memory_chunks, 64), generator=gen),
                        torch.full((memory_chunks,), 64, dtype=torch.int32), batch_chunks=256)
    rows = 64
    engine.set_namespace(torch.zeros(rows, dtype=torch.int32), torch.full((rows,), memory_chunks, dtype=torch.int32))
    tok = engine.prefill(torch.randint(0, cfg.vocab_size, (rows, 4096), generator=gen),
                         torch.full((rows,), 4096, dtype=torch.int32), 16, row_batch=4).float().argmax(-1)
    tok = engine.decode_step(tok).float().argmax(-1)
    engine.capture_decode()
    for _ in range(3):
        tok = engine.decode_step_graphed(tok).float().argmax(-1)
    tp.barrier()
    t0 = time.perf_counter()
    for _ in range(5):
        tok = engine.decode_step_graphed(tok).float().argmax(-1)
    torch.cuda.synchronize()
    if tp.rank == 0:
        print(f"step wall ms {1000 * (time.perf_counter() - t0) / 5:.2f}")
    tp.barrier()
    # every rank runs under the profiler (its start-up stalls the host), only rank 0 prints
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        tp.barrier()
        engine.decode_step_graphed(tok)
        torch.cuda.synchronize()
    if tp.rank == 0:
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=40, max_name_column_width=70))
    tp.barrier()
    engine.release_graph()
    tp.close()
    dist.destroy_process_group()


def attention_fwd(iters: int = 20) -> None:
    """Device time of the forward attention kernels (tcgen05 and mma.sync) on the shapes the
    training step and the Llama prefill run: CUDA events around ``iters`` back-to-back
    launches, median of five such batches."""
    import math
    import statistics

    from .ops._ext import require

    ext = require()
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    shapes = [  # name, B, T, H, Hkv, D, memory keys per row
        ("tinygpt prompt", 8, 1024, 12, 12, 64, 1024),
        ("tinygpt chunk encode", 128, 64, 12, 12, 64, 256),
        ("llama prefill 4k", 1, 4096, 32, 8, 128, 1024),
        ("llama chunk encode", 64, 64, 32, 8, 128, 0),
    ]
    print(f"{'shape':24s} {'impl':8s} {'us':>9s} {'TFLOP/s':>8s}")
    for name, B, T, H, Hkv, D, M in shapes:
        q = torch.randn((B, T, H * D), generator=gen, device=dev).bfloat16()
        k = torch.randn((B, T, Hkv * D), generator=gen, device=dev).bfloat16()
        v = torch.randn((B, T, Hkv * D), generator=gen, device=dev).bfloat16()
        pool = torch.randn((max(M, 1) * 4, 2 * Hkv * D), generator=gen, device=dev).bfloat16()
        idx = torch.randint(0, pool.shape[0], (B, max(M, 1)), generator=gen, device=dev, dtype=torch.int32)
        mlen = torch.full((B,), M, device=dev, dtype=torch.int32)
        keys = B * H * (M * T + T * (T + 1) / 2)
        flops = 4.0 * D * keys
        for impl in ("tcgen05", "mma"):
            ext.set_attention_impl(impl)
            call = lambda: ext.attention_fwd(q, k, v, H, Hkv, D, pool[:, :Hkv * D], pool[:, Hkv * D:], idx, mlen,
                                             None, 1.0 / math.sqrt(D))
            for _ in range(3):
                call()
            times = []
            for _ in range(5):  # five batches of `iters` back-to-back launches
                a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(iters):
                    call()
                b_.record()
                b_.synchronize()
                times.append(a.elapsed_time(b_) * 1000 / iters)
            us = statistics.median(times)
            print(f"{name:24s} {impl:8s} {us:9.1f} {flops / us / 1e6:8.1f}")
    ext.set_attention_impl("tcgen05")


def sweep_table(tokens: int = 1 << 24, gists: int = 1, k: int = 16) -> None:
    """Kernel table of one fused layer step of the memory sweep (one GPU, 16M-token memory)."""
    from .inference.memory_sweep import HEAD_DIM, HEADS, KV_DIM, ShardedLayerMemory, fused_layer_step

    dev = torch.device("cuda", 0)
    mem = ShardedLayerMemory(tokens, gists, dev)
    gen = torch.Generator(device=dev).manual_seed(3)
    rq = torch.randn((64, KV_DIM), generator=gen, device=dev)
    q = torch.randn((64, HEADS * HEAD_DIM), generator=gen, device=dev).to(torch.bfloat16)
    for _ in range(3):
        fused_layer_step(mem, rq, q, k)
    torch.cuda.synchronize()
    _table(lambda: fused_layer_step(mem, rq, q, k), rows=15)


def decode_attention_sweep(iters: int = 20) -> None:
    """Device time of one Llama-3-8B layer's decode attention (64 rows, 4,352-slot local caches with
    4,096 + a few keys, 16 routed 64-token chunks per row; K/V > the L2) for the TMA-fed kernel at
    2 / 3 / 4 pipeline stages and split sizes 512 / 1024, and the cp.async kernel."""
    from .ops import _ext

    ext = _ext.require()
    dev = torch.device("cuda", 0)
    B, H, Hkv, D, max_len, chunks = 64, 32, 8, 128, 4352, 4096
    gen = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(B, H * D, device=dev, generator=gen).bfloat16()
    pool = torch.randn(chunks * 64, 2 * Hkv * D, device=dev, generator=gen).bfloat16()
    cache = torch.randn(2, B, max_len, Hkv * D, device=dev, generator=gen).bfloat16()
    picks = torch.stack([torch.randperm(chunks, device=dev)[:16] for _ in range(B)])
    mem_idx = (picks[:, :, None] * 64 + torch.arange(64, device=dev)).reshape(B, -1).to(torch.int32).contiguous()
    mem_len = torch.full((B,), 1024, device=dev, dtype=torch.int32)
    loc_len = torch.full((B,), 4100, device=dev, dtype=torch.int32)
    nbytes = B * Hkv * (1024 + 4100) * D * 2 * 2
    rows = []
    configs = [("cp.async", False, 3, 512)] + [(f"tma s{st} split{sp}", True, st, sp) for st in (2, 3)
                                               for sp in (512, 1024, 2048)]
    for name, tma, stages, split in configs:
        ext.decode_set_tma(tma)
        ext.decode_set_stages(stages)
        args = (q, H, Hkv, D, pool[:, : Hkv * D], pool[:, Hkv * D:], mem_idx, mem_len, cache[0], cache[1], loc_len,
                1024 + max_len, split, False)
        for _ in range(3):
            ext.decode_attention(*args)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            ext.decode_attention(*args)
        e.record()
        torch.cuda.synchronize()
        us = 1000 * s.elapsed_time(e) / iters
        rows.append((name, us, nbytes / us / 1e6))
    ext.decode_set_tma(True)
    ext.decode_set_stages(2)
    for name, us, tbs in rows:
        print(f"{name:20s} {us:8.1f} us  {tbs:5.2f} TB/s (attention + split merge, {nbytes / 1e9:.2f} GB of K/V)")


def decode_overlap_probe(iters: int = 20) -> None:
    """One Llama-3-8B layer's routing + decode attention (64 rows, 4,096 chunks of 1,024-wide gists,
    top-16, 4,100 local keys per row; K/V > the L2), serial (scores, top-k, one attention launch)
    against overlapped (local splits on the current stream while a high-priority side stream
    scores, selects and attends over the memory splits; then the merge), and the attention
    phases alone."""
    import torch.nn.functional as F

    from .ops import _ext

    ext = _ext.require()
    dev = torch.device("cuda", 0)
    B, H, Hkv, D, max_len, chunks, W = 64, 32, 8, 128, 4352, 4096, 1024
    gen = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(B, H * D, device=dev, generator=gen).bfloat16()
    pool = torch.randn(chunks * 64, 2 * Hkv * D, device=dev, generator=gen).bfloat16()
    mk, mv = pool[:, : Hkv * D], pool[:, Hkv * D:]
    cache = torch.randn(2, B, max_len, Hkv * D, device=dev, generator=gen).bfloat16()
    loc_len = torch.full((B,), 4100, device=dev, dtype=torch.int32)
    gists = F.normalize(torch.randn(chunks, W, device=dev, generator=gen), dim=-1)
    gists_bf = gists.bfloat16().contiguous()
    rq = torch.randn(B, W, device=dev, generator=gen).bfloat16()
    lo = torch.zeros(B, dtype=torch.int32, device=dev)
    hi = torch.full((B,), chunks, dtype=torch.int32, device=dev)
    clen = torch.full((chunks,), 64, dtype=torch.int32, device=dev)
    row0 = torch.arange(chunks, dtype=torch.int32, device=dev) * 64
    scores = torch.empty(B, chunks, device=dev)
    sk, msk = 1024, int(os.environ.get("PRA_PROBE_MEM_SPLIT", "256"))
    n_mem, n_loc = 1024 // msk, -(-max_len // sk)
    part_o = torch.empty(B, H, n_mem + n_loc, D, device=dev)
    part_ml = torch.empty(B, H, n_mem + n_loc, 2, device=dev)
    side = torch.cuda.Stream(dev, priority=-1)
    common = dict(mem_splits=n_mem, mem_split_keys=msk, part_o=part_o, part_ml=part_ml)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    local_ctas = int(os.environ.get("PRA_PROBE_LOCAL_CTAS", str(2 * sms)))  # persistent local grid

    def route():
        ext.decode_gemm(rq, gists_bf, None, None, scores, None, 0, 0, [], [], 0, None, 0, None)
        return ext.route_topk(scores, rq, gists, lo, hi, clen, row0, 16, 64, -1, 1024, False, 0, 1, 1)

    def serial():
        mem_idx, mem_len, _ = route()
        ext.decode_attention(q, H, Hkv, D, mk, mv, mem_idx, mem_len, cache[0], cache[1], loc_len, 1024 + max_len,
                             sk, False)

    def overlapped():
        main = torch.cuda.current_stream()
        side.wait_stream(main)
        ext.decode_attention(q, H, Hkv, D, None, None, None, None, cache[0], cache[1], loc_len, 0, sk, False,
                             split_lo=n_mem, split_count=n_loc, phase=1, max_ctas=local_ctas, **common)
        with torch.cuda.stream(side):
            ext.set_launch_priority(True)
            mem_idx, mem_len, _ = route()
            ext.decode_attention(q, H, Hkv, D, mk, mv, mem_idx, mem_len, cache[0], cache[1], loc_len, 0, sk, False,
                                 split_lo=0, split_count=n_mem, phase=1, **common)
            ext.set_launch_priority(False)
        main.wait_stream(side)
        ext.decode_attention(q, H, Hkv, D, None, None, None, None, cache[0], cache[1], loc_len, 0, sk, False,
                             phase=2, **common)

    mem_idx0, mem_len0, _ = route()

    def local_only():
        ext.decode_attention(q, H, Hkv, D, None, None, None, None, cache[0], cache[1], loc_len, 0, sk, False,
                             split_lo=n_mem, split_count=n_loc, phase=1, max_ctas=local_ctas, **common)

    def memory_only():
        ext.decode_attention(q, H, Hkv, D, mk, mv, mem_idx0, mem_len0, cache[0], cache[1], loc_len, 0, sk, False,
                             split_lo=0, split_count=n_mem, phase=1, **common)

    def single():
        ext.decode_attention(q, H, Hkv, D, mk, mv, mem_idx0, mem_len0, cache[0], cache[1], loc_len, 1024 + max_len,
                             sk, False)

    for name, fn in (("routing only", route), ("single attention launch", single), ("local splits", local_only),
                     ("memory splits", memory_only), ("serial routing + attention", serial),
                     ("overlapped routing + attention", overlapped)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        print(f"{name:32s} {1000 * s.elapsed_time(e) / iters:8.1f} us (memory split {msk} keys, local grid "
              f"{local_ctas or 'full'})")


def route_topk_bench(iters: int = 50) -> None:
    """Device time of the exact top-k routing kernel for the decode shapes: 64 query rows,
    2,048 / 4,096 / 8,192 chunks per rank, 1,024-wide gists, top-16 from 64 candidates."""
    import torch.nn.functional as F

    from .ops import _ext

    ext = _ext.require()
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    for n in (2048, 4096, 8192):
        gists = F.normalize(torch.randn(n, 1024, device=dev, generator=gen), dim=-1)
        query = torch.randn(64, 1024, device=dev, generator=gen)
        scores = (F.normalize(query, dim=-1).bfloat16().float() @ gists.bfloat16().float().t()).contiguous()
        lo = torch.zeros(64, dtype=torch.int32, device=dev)
        hi = torch.full((64,), n, dtype=torch.int32, device=dev)
        clen = torch.full((n,), 64, dtype=torch.int32, device=dev)
        row0 = torch.arange(n, dtype=torch.int32, device=dev) * 64

        def call():
            ext.route_topk(scores, query, gists, lo, hi, clen, row0, 16, 64, -1, 1024, False, 0, 1, 1)

        for _ in range(3):
            call()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            call()
        e.record()
        torch.cuda.synchronize()
        trace = torch.zeros(8, dtype=torch.int64, device=dev)
        ext.route_topk(scores, query, gists, lo, hi, clen, row0, 16, 64, -1, 1024, False, 0, 1, 1, -1, None, trace)
        torch.cuda.synchronize()
        t = trace.tolist()
        phases = [t[i + 1] - t[i] for i in range(4)]
        print(f"route_topk 64 rows x {n} chunks: {1000 * s.elapsed_time(e) / iters:.1f} us; CTA 0 cycles: radix "
              f"{phases[0]}, candidates {phases[1]}, rescoring {phases[2]}, selection {phases[3]}")


def decode_gemm_sweep(iters: int = 30) -> None:
    """Device time of the decode GEMM (64 token rows) on the Llama-3-8B projection shapes of one
    GPU and of tensor-parallel shards (2 and 8 ranks), for one or two CTAs per SM and the fewest
    K blocks a split keeps; weights > the L2 are rotated between launches."""
    from .ops import _ext

    ext = _ext.require()
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    shapes = {"qkv tp1": (7168, 4096), "o tp1": (4096, 4096), "gate_up tp1": (28672, 4096), "down tp1": (4096, 14336),
              "qkv tp8": (1792, 4096), "o tp8": (4096, 512), "gate_up tp8": (3584, 4096), "down tp8": (4096, 1792)}
    configs = [(1, 8, 8), (2, 8, 8), (2, 8, 4), (2, 8, 2), (2, 4, 4)]
    print("shape            " + "  ".join(f"ctas{c}/minkb{k}/max{m}" for c, k, m in configs))
    for name, (n, k) in shapes.items():
        copies = max(2, int(2 * 128e6 // (n * k * 2)) + 1)  # > L2 in total
        ws = [(torch.randn(n, k, device=dev, generator=gen) * 0.02).bfloat16() for _ in range(copies)]
        x = torch.randn(64, k, device=dev, generator=gen).bfloat16()
        out = torch.empty(64, n, device=dev, dtype=torch.bfloat16)
        cells = []
        for ctas, min_kb, max_splits in configs:
            ext.decode_gemm_configure(ctas, min_kb, max_splits)
            for w in ws:
                ext.decode_gemm(x, w, None, None, out, None, 0, 0, [], [], 0, None, 0, None)
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for i in range(iters):
                ext.decode_gemm(x, ws[i % copies], None, None, out, None, 0, 0, [], [], 0, None, 0, None)
            e.record()
            torch.cuda.synchronize()
            us = 1000 * s.elapsed_time(e) / iters
            cells.append(f"{us:6.1f}us {n * k * 2 / us / 1e6:4.2f}TB/s")
        print(f"{name:16s} " + "  ".join(cells))
    ext.decode_gemm_configure(2, 8, 8)


def decode_gemm_one(iters: int = 4) -> None:
    """A few launches of one decode GEMM (64 token rows x the Llama-3-8B QKV weight with the
    routing-query rows, 7,168 x 4,096 bf16 = 58.7 MB, above nothing but the L2 of a previous
    launch's other copy): the small case for a full profiler capture of ``decode_gemm_kernel``."""
    from .ops import _ext

    ext = _ext.require()
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    n, k = 7168, 4096
    ws = [(torch.randn(n, k, device=dev, generator=gen) * 0.02).bfloat16() for _ in range(3)]  # 176 MB > L2
    x = torch.randn(64, k, device=dev, generator=gen).bfloat16()
    out = torch.empty(64, n, device=dev, dtype=torch.bfloat16)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for i in range(iters):
        ext.decode_gemm(x, ws[i % 3], None, None, out, None, 0, 0, [], [], 0, None, 0, None)
    e.record()
    torch.cuda.synchronize()
    ref = x.float() @ ws[(iters - 1) % 3].float().t()
    err = (out.float() - ref).abs().max().item()
    print(f"decode_gemm 64x{n}x{k}: {1000 * s.elapsed_time(e) / iters:.1f} us per launch (incl. first), max err {err:.3g}")


def gemm_train_shapes(iters: int = 20) -> None:
    """Device time of this library's training GEMMs (CUTLASS sm100 tcgen05 kernels behind
    ``ext.gemm``) against cuBLAS through torch on the TinyGPT-PRA-163M shapes: prompt rows
    8,192, cache-encode rows 16,384, d_model 768, MLP 3,072, vocabulary 50,304."""
    from .ops import _ext

    ext = _ext.require()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape):
        return (torch.randn(*shape, device=dev, generator=g) * 0.05).bfloat16()

    def timed(fn):
        for _ in range(3):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        return 1000 * s.elapsed_time(e) / iters

    print(f"{'shape':44s} {'ours us':>8s} {'cuBLAS us':>9s} {'ours TF/s':>9s} {'ratio':>6s}")
    for m in (8192, 16384):
        for name, n, k in (("qkv", 2304, 768), ("o", 768, 768), ("fc1", 3072, 768), ("fc2", 768, 3072)):
            a, w, bias = rnd(m, k), rnd(n, k), rnd(n)
            d = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
            ours = timed(lambda: ext.gemm("tn", a, w, None, d, bias, None, 1.0, 0.0, None))
            ref = timed(lambda: torch.nn.functional.linear(a, w, bias))
            fl = 2 * m * n * k
            print(f"{'fwd ' + name + f' {m}x{n}x{k}':44s} {ours:8.1f} {ref:9.1f} {fl / ours / 1e6:9.0f} {ref / ours:6.2f}")
            if name == "fc1":  # + GELU epilogue storing the pre-activation too, against linear + gelu
                z = torch.empty_like(d)
                ours = timed(lambda: ext.gemm("tn_gelu", a, w, None, d, bias, z, 1.0, 0.0, None))
                ref = timed(lambda: torch.nn.functional.gelu(torch.nn.functional.linear(a, w, bias)))
                print(f"{'fwd fc1+gelu' + f' {m}x{n}x{k}':44s} {ours:8.1f} {ref:9.1f} {fl / ours / 1e6:9.0f} "
                      f"{ref / ours:6.2f}")
            if name == "fc2" and m == 8192:  # dgrad through fc2 with the GELU derivative of fc1's output
                dy2, z1 = rnd(m, n), rnd(m, k)
                dz = torch.empty(m, k, device=dev, dtype=torch.bfloat16)
                ours = timed(lambda: ext.gemm("nn_dgelu", dy2, w, None, dz, None, z1, 1.0, 0.0, None))
                ref = timed(lambda: dy2 @ w)
                print(f"{'dgrad fc2+dgelu' + f' {m}x{k}x{n}':44s} {ours:8.1f} {ref:9.1f} {fl / ours / 1e6:9.0f} "
                      f"{ref / ours:6.2f}")
            if m == 8192:
                dy = rnd(m, n)
                dx = torch.empty(m, k, device=dev, dtype=torch.bfloat16)
                ours = timed(lambda: ext.gemm("nn", dy, w, None, dx, None, None, 1.0, 0.0, None))
                ref = timed(lambda: dy @ w)
                print(f"{'dgrad ' + name + f' {m}x{k}x{n}':44s} {ours:8.1f} {ref:9.1f} {fl / ours / 1e6:9.0f} {ref / ours:6.2f}")
                dw = torch.empty(n, k, device=dev, dtype=torch.bfloat16)
                ours = timed(lambda: ext.gemm("wgrad", dy, a, None, dw, None, None, 1.0, 0.0, None))
                ref = timed(lambda: dy.t() @ a)
                print(f"{'wgrad ' + name + f' {n}x{k}x{m}':44s} {ours:8.1f} {ref:9.1f} {fl / ours / 1e6:9.0f} {ref / ours:6.2f}")
    m, v, k = 8192, 50304, 768
    a, w = rnd(m, k), rnd(v, k)
    d = torch.empty(m, v, device=dev, dtype=torch.bfloat16)
    fl = 2 * m * v * k
    ours = timed(lambda: ext.gemm("tn", a, w, None, d, None, None, 1.0, 0.0, None))
    ref = timed(lambda: a @ w.t())
    print(f"{'fwd lm_head ' + f'{m}x{v}x{k}':44s} {ours:8.1f} {ref:9.1f} {fl / ours / 1e6:9.0f} {ref / ours:6.2f}")
    dx = torch.empty(m, k, device=dev, dtype=torch.bfloat16)
    ours = timed(lambda: ext.gemm("nn", d, w, None, dx, None, None, 1.0, 0.0, None))
    ref = timed(lambda: d @ w)
    print(f"{'dgrad lm_head ' + f'{m}x{k}x{v}':44s} {ours:8.1f} {ref:9.1f} {fl / ours / 1e6:9.0f} {ref / ours:6.2f}")
    dw = torch.empty(v, k, device=dev, dtype=torch.bfloat16)
    ours = timed(lambda: ext.gemm("wgrad", d, a, None, dw, None, None, 1.0, 0.0, None))
    ref = timed(lambda: d.t() @ a)
    print(f"{'wgrad lm_head ' + f'{v}x{k}x{m}':44s} {ours:8.1f} {ref:9.1f} {fl / ours / 1e6:9.0f} {ref / ours:6.2f}")


CASES = {"attention-fwd": attention_fwd, "decode-gemm-one": decode_gemm_one, "gemm-train-shapes": gemm_train_shapes,
         "decode-overlap-probe": decode_overlap_probe, "sweep-table": sweep_table, "train-small": train_small, "decode-small": decode_small, "train-table": train_table,
         "decode-table": decode_table, "decode-table-tp": decode_table_tp,
         "decode-attention-sweep": decode_attention_sweep, "route-topk-bench": route_topk_bench,
         "decode-gemm-sweep": decode_gemm_sweep}


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("case", choices=sorted(CASES))
    args = parser.parse_args(argv)
    if args.case != "decode-table-tp":
        torch.cuda.set_device(0)
    CASES[args.case]()


if __name__ == "__main__":
    main()
