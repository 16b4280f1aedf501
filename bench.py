"""TinyGPT-PRA training throughput (tokens/s) on one node, one rank per GPU.

Workload (fixed per GPU, weak scaling): TinyGPT-PRA ~125M (12 PRA layers,
d_model 768, 12 heads, native context 1024, GPT-2-size vocabulary 50257),
bf16.  Each example's prompt holds 2 root references; each root names 1
child, which names 6 leaves (16 references per example, depth-2 child-first
recursion, 128 uniform-random tokens each), chunks of 64 tokens with 2 k-means
gists per chunk; routing keeps 2 references x 2 chunks (256 memory tokens) next
to a 768-token direct window.  Every step rebuilds every row's cache (the
reference semantics), runs the routed forward, backward and AdamW.  Synthetic
data, random-initialised weights.  Per-step working set (weights + activations)
is far larger than the 126 MB L2, so no explicit flush is needed.

``--impl reference`` runs the unmodified reference (installed in baseline/_ref)
through its own batch step and optimizer code on the same data; with more than
one rank its gradients are averaged with NCCL.

Launch: ``python bench.py`` (1 GPU) or ``torchrun --nproc-per-node N bench.py --gpus N``.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PER_GPU_BATCH = 8
VOCAB = 50257
MODEL = dict(d_model=768, n_heads=12, n_layers=12, max_seq_len=1024, model_variant="td_pra", chunking_mode="fixed",
             fixed_chunk_tokens=64, top_k_references=2, top_k_chunks_per_reference=2, gist_mode="kmeans",
             gists_per_chunk=2, recursive_refs_enabled=True, recursive_max_depth=2, trigger_threshold=-1.0)
# Written under the hierarchical stage name both frameworks' dataset registries know.
STAGE = "stage1_hierarchical_synthetic"
TREE = dict(roots=2, children=1, grandchildren=6, doc_tokens=128, prompt_tokens=767, vocab=VOCAB)


def _env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(tempfile.mkstemp(suffix=".csv")[1])

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self) -> dict:
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({name for r in rows for name, flag in zip(names, r[5:9]) if flag.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


def _make_data(root: Path, examples: int, seed: int, tokenizer) -> None:
    """Write the stage and register every reference handle it uses (fixes the vocabulary size)."""
    from pdattention_b200.data.datasets import read_jsonl
    from pdattention_b200.data.generators import generate_hierarchical_tokens

    stage = generate_hierarchical_tokens(root / STAGE, examples=examples, seed=seed, **TREE)
    for name in ("documents.jsonl", "questions.jsonl"):
        for row in read_jsonl(stage / name):
            tokenizer.encode(row.get("text") or row.get("prompt") or "")


def _loader(module_cls, root: Path, tokenizer, rank: int, world: int):
    kwargs = dict(batch_size=PER_GPU_BATCH, max_seq_len=MODEL["max_seq_len"], tokenizer=tokenizer, shuffle=False,
                  pin_memory=torch.cuda.is_available())
    if "rank" in module_cls.__init__.__code__.co_varnames:
        kwargs.update(rank=rank, world_size=world)
    return module_cls(STAGE, str(root), **kwargs).load()


def _batches(dm, rank: int, world: int, count: int):
    """``count`` batches of this rank's disjoint shard (cycled)."""
    dataset = dm.dataset
    per_rank = [dataset[i] for i in range(rank, len(dataset), world)]
    out = []
    i = 0
    while len(out) < count:
        rows = [per_rank[(i + j) % len(per_rank)] for j in range(PER_GPU_BATCH)]
        batch = dm.collator(rows)
        if torch.cuda.is_available():
            for key in ("input_ids", "labels", "attention_mask"):
                batch[key] = batch[key].pin_memory()
        out.append(batch)
        i += PER_GPU_BATCH
    return out


def _sync_all(world: int) -> None:
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[torch.cuda.current_device()])
        torch.cuda.synchronize()


def _max(value: float, world: int) -> float:
    if world <= 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _gather(value: float, world: int) -> list[float]:
    """Every rank's value (rank order); collective, so every rank calls it."""
    if world <= 1:
        return [value]
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def run(impl: str, steps: int, warmup: int, gpus: int, reference_autocast: bool = False) -> dict:
    rank, local, world = _env()
    if gpus != world:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    from pdattention_b200.data import WordIdTokenizer

    tmp = Path(tempfile.mkdtemp(prefix=f"pra_bench_{rank}_"))
    total_steps = steps + warmup
    tokenizer = WordIdTokenizer(VOCAB)
    _make_data(tmp, examples=max(PER_GPU_BATCH * world * 2, 32), seed=0, tokenizer=tokenizer)
    if impl == "reference":
        step_fn, model_desc, counter = _reference_arm(tmp, tokenizer, rank, world, reference_autocast)
    else:
        step_fn, model_desc, counter = _pra_arm(tmp, tokenizer, rank, world)
    batches = step_fn.batches(total_steps)
    tokens_per_step = [int(b["attention_mask"].sum()) for b in batches]

    def upcoming(i):
        return batches[i + 1] if i + 1 < total_steps else None

    for i in range(warmup):
        step_fn(batches[i], upcoming(i))
    _sync_all(world)
    if counter is not None:
        counter.reset()
        counter.enabled = True
    start_evt, end_evt = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d = d2h = 0
    with ClockSampler(local) as clocks:
        _sync_all(world)
        wall0 = time.perf_counter()
        start_evt.record()
        host_s = 0.0
        for i in range(warmup, total_steps):
            t_host = time.perf_counter()
            loss_host, moved, read = step_fn(batches[i], upcoming(i))
            host_s += time.perf_counter() - t_host
            h2d += moved
            d2h += read
        if step_fn.flush is not None:
            loss_host = step_fn.flush()
        end_evt.record()
        _sync_all(world)
        wall = time.perf_counter() - wall0
    if counter is not None:
        counter.enabled = False
    per_rank_device = _gather(start_evt.elapsed_time(end_evt) / 1000.0, world)
    per_rank_host = _gather(host_s, world)
    device_s = max(per_rank_device)
    wall_s = _max(wall, world)
    local_tokens = sum(tokens_per_step[warmup:])
    total_tokens = local_tokens * world  # identical shards sizes on every rank
    result = {
        "metric": "PRA train tokens/s (TinyGPT-PRA ~125M, data parallel)",
        "value": total_tokens / device_s,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": 1000.0 * device_s / steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if impl != "reference" else ("bf16-autocast" if reference_autocast else "fp32"),
        "data": "synthetic (seeded uniform-random token ids, depth-2 recursive references), random-init weights",
        "config": {"model": model_desc, "global_batch": PER_GPU_BATCH * world, "seq_len": MODEL["max_seq_len"],
                   "direct_tokens_per_row": TREE["prompt_tokens"] + 1, "references_per_row": 16,
                   "chunk_tokens": 64, "gists_per_chunk": 2, "parallelism": f"dp{world}",
                   "dp_reduction": ("fused peer-memory all-reduce kernel" if impl != "reference" and world > 1
                                    else "nccl all-reduce" if world > 1 else "none"),
                   "l2": "per-step working set exceeds the 126 MB L2 (no flush)"},
        "clocks": clocks.summary(),
        "e2e": {"value": total_tokens / wall_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d // max(steps, 1),
                "d2h_bytes_per_step": d2h // max(steps, 1)},
        "gpu_launches": (counter.launches if counter is not None else 0),
        "host_ms_per_step": 1000.0 * max(per_rank_host) / steps,  # time inside the step call on the host
        "per_rank_ms_per_step": {"device": [round(1000.0 * v / steps, 3) for v in per_rank_device],
                                 "host": [round(1000.0 * v / steps, 3) for v in per_rank_host]},
        "last_loss": loss_host,
    }
    if impl == "reference":
        result["impl"] = "reference"
    step_fn.close()
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return result


class _Step:
    def __init__(self, fn, batch_source, close=None, flush=None):
        self.fn = fn
        self.batches = batch_source
        self.close = close or (lambda: None)
        self.flush = flush  # returns the last step's host-read result, if reads lag one step

    def __call__(self, batch, next_batch=None):
        return self.fn(batch, next_batch)


def _moved_bytes(batch) -> int:
    return sum(batch[k].numel() * batch[k].element_size() for k in ("input_ids", "labels", "attention_mask"))


def _pra_arm(root: Path, tokenizer, rank: int, world: int):
    from pdattention_b200.config import PRAConfig, ResolverServiceConfig, TrainConfig
    from pdattention_b200.data import PRADataModule
    from pdattention_b200.models.fastpath import prepare_model
    from pdattention_b200.ops._ext import launch_counter
    from pdattention_b200.parallel.dp import attach_data_parallel
    from pdattention_b200.pra_train import training_step

    dm = _loader(PRADataModule, root, tokenizer, rank, world)
    torch.manual_seed(0)
    cfg = PRAConfig(vocab_size=tokenizer.vocab_size, device="cuda", **MODEL)
    model = prepare_model(cfg, "cuda")
    if getattr(model, "_device_runtime", None) is None:
        raise RuntimeError("device path unavailable for the benchmark config")
    model.train()
    optimizer = model.build_optimizer(TrainConfig(device="cuda", learning_rate=3e-4))
    reducer = attach_data_parallel(model, optimizer, world)
    resolver = ResolverServiceConfig()
    # The loss of step i is copied to pinned host memory on the stream and read after step
    # i + 1 has been queued, so the host never waits for the GPU between steps.
    host_loss = [torch.zeros((), dtype=torch.float32).pin_memory() for _ in range(2)]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    pending = {"slot": None, "value": float("nan")}

    def read_pending():
        slot = pending["slot"]
        if slot is not None:
            done[slot].synchronize()
            pending["value"] = float(host_loss[slot])
            pending["slot"] = None
        return pending["value"]

    def step(batch, next_batch=None):
        dev_batch = dict(batch)
        for key in ("input_ids", "labels", "attention_mask"):
            dev_batch[key] = batch[key].to("cuda", non_blocking=True)
        loss, _ = training_step(model, dev_batch, "cuda", tokenizer, optimizer, resolver_config=resolver,
                                next_batch=next_batch)
        previous = read_pending()
        slot = 0 if pending.get("last", 1) == 1 else 1
        pending["last"] = slot
        host_loss[slot].copy_(loss.detach().float(), non_blocking=True)
        done[slot].record()
        pending["slot"] = slot
        return previous, _moved_bytes(batch), 4

    params = sum(p.numel() for p in model.parameters())
    def close():
        if reducer is not None:
            reducer.check()  # raises if a peer wait timed out during the run
            if hasattr(reducer, "close"):
                reducer.close()

    return (_Step(step, lambda n: _batches(dm, rank, world, n), close, read_pending),
            f"TinyGPT-PRA-{params / 1e6:.0f}M", launch_counter())


def _reference_arm(root: Path, tokenizer, rank: int, world: int, autocast: bool = False):
    """The unmodified reference: its data module, model, ``_pra_batch_step``, ``grad_norm`` and
    stock AdamW.  ``autocast`` runs the same step under ``torch.autocast(bfloat16)`` (an optional
    variant that separates the precision share of the gap from the engineering share)."""
    ref_root = REPO / "baseline" / "_ref"
    if not (ref_root / "pra_torch").exists():
        raise _Unavailable("reference not installed in baseline/_ref")
    sys.path.append(str(ref_root))
    from common.metrics import grad_norm as ref_grad_norm  # reference modules
    from data.datamodules import PRADataModule as RefDataModule
    from pra_torch.config import CacheServiceConfig, PRAConfig as RefConfig, ResolverServiceConfig
    from pra_torch.model import TinyPRAModel as RefModel
    from pra_torch.pra_train import _pra_batch_step as ref_batch_step

    dm = _loader(RefDataModule, root, tokenizer, rank, world)
    torch.manual_seed(0)
    cfg = RefConfig(vocab_size=tokenizer.vocab_size, device="cuda", **MODEL)
    model = RefModel(cfg).to("cuda").train()
    optimizer = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.0)
    resolver, cache = ResolverServiceConfig(), CacheServiceConfig()
    params = [p for p in model.parameters()]

    def step(batch, next_batch=None):
        optimizer.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            loss, _ = ref_batch_step(model, batch, "cuda", tokenizer, resolver, cache)
        loss.backward()
        if world > 1:
            import torch.distributed as dist

            grads = [p.grad for p in params if p.grad is not None]
            flat = torch.cat([g.reshape(-1) for g in grads])
            dist.all_reduce(flat)
            flat /= world
            offset = 0
            for g in grads:
                g.copy_(flat[offset: offset + g.numel()].view_as(g))
                offset += g.numel()
        ref_grad_norm(model.parameters())
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        optimizer.step()
        return float(loss.detach().cpu()), _moved_bytes(batch), 4

    n = sum(p.numel() for p in model.parameters())
    precision = "bf16 autocast" if autocast else "fp32"
    return _Step(step, lambda k: _batches(dm, rank, world, k)), f"TinyGPT-PRA-{n / 1e6:.0f}M (reference {precision})", None


def run_decode(impl: str, steps: int, warmup: int, gpus: int, memory_tokens: int | None, batch: int) -> dict:
    """PRA decode on a Llama-3-8B-architecture model (random weights) with a shared chunk memory.

    ``impl="reference"``: the reference has no Llama-family PRA model, no tensor parallelism
    and no 8B decode path, so the comparison arm is ``baseline/torch_pra_decode.py``, the
    reference's PRA decode semantics in plain PyTorch + cuBLAS + NCCL (it imports nothing
    from this framework), on the same workload."""
    if impl == "reference":
        return _run_decode_torch_arm(steps, warmup, gpus, memory_tokens, batch)
    rank, local, world = _env()
    if gpus != world:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    tp = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        from pdattention_b200.parallel.tp import TensorParallel

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        tp = TensorParallel()
    from pdattention_b200.inference.decode_bench import run_decode_benchmark
    from pdattention_b200.ops._ext import launch_counter

    tokens = memory_tokens or (1 << 20 if world > 1 else 1 << 18)
    refs = 32
    counter = launch_counter()
    clocks = ClockSampler(local)
    out = run_decode_benchmark(batch=batch, refs=refs, ref_tokens=tokens // refs, steps=steps, warmup=warmup, tp=tp,
                               clocks=clocks, counter=counter)
    result = {
        "metric": "PRA decode tokens/s (Llama-3-8B architecture, sharded chunk memory)",
        "value": out["tokens_per_s"],
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": out["tpot_p50_ms"],
        "tpot_p50_ms": out["tpot_p50_ms"],
        "tpot_p90_ms": out["tpot_p90_ms"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (uniform-random token ids for prompts and references), random-init weights",
        "config": {"model": f"Llama-3-8B architecture ({out['params_b']:.2f}B params)", "global_batch": batch,
                   "seq_len": out["prompt_tokens"], "memory_tokens": out["memory_tokens"],
                   "chunk_tokens": out["chunk_tokens"], "gists_per_chunk": 1, "chunk_top_k": out["top_k_chunks"],
                   "parallelism": f"tp{world}", "memory_gb_per_gpu": round(out["memory_gb_per_gpu"], 2),
                   "build_tokens_per_s": out["build_tokens_per_s"], "prefill_tokens_per_s": out["prefill_tokens_per_s"],
                   "l2": "per-step working set (weights, caches, memory) exceeds the 126 MB L2 (no flush)"},
        "clocks": clocks.summary(),
        "e2e": {"value": out["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": out["h2d_bytes_per_step"],
                "d2h_bytes_per_step": out["d2h_bytes_per_step"]},
        "gpu_launches": out["gpu_launches"],
    }
    if tp is not None:
        tp.close()
        import torch.distributed as dist

        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return result


def _run_decode_torch_arm(steps: int, warmup: int, gpus: int, memory_tokens: int | None, batch: int) -> dict:
    rank, local, world = _env()
    if gpus != world:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    sys.path.insert(0, str(REPO / "baseline"))
    import torch_pra_decode

    tokens = memory_tokens or (1 << 20 if world > 1 else 1 << 18)
    clocks = ClockSampler(local)
    with clocks:
        out = torch_pra_decode.run(batch=batch, memory_tokens=tokens, steps=steps, warmup=warmup)
    result = {
        "metric": "PRA decode tokens/s (Llama-3-8B architecture, sharded chunk memory)", "value": out["tokens_per_s"],
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": out["tpot_p50_ms"],
        "tpot_p50_ms": out["tpot_p50_ms"], "tpot_p90_ms": out["tpot_p90_ms"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform-random token ids for prompts and references), random-init weights",
        "config": {"model": "Llama-3-8B architecture", "global_batch": batch, "seq_len": out["prompt_tokens"],
                   "memory_tokens": out["memory_tokens"], "chunk_tokens": 64, "gists_per_chunk": 1,
                   "chunk_top_k": out["top_k_chunks"], "parallelism": f"tp{world}",
                   "build_tokens_per_s": out["build_tokens_per_s"],
                   "prefill_tokens_per_s": out["prefill_tokens_per_s"]},
        "clocks": clocks.summary(),
        "e2e": {"value": out["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": out["h2d_bytes_per_step"],
                "d2h_bytes_per_step": out["d2h_bytes_per_step"]},
        "gpu_launches": 0, "impl": "reference",
        "reference_kind": "the reference's PRA decode semantics in plain PyTorch + cuBLAS + NCCL "
                          "(baseline/torch_pra_decode.py); the reference itself has no Llama-family or TP path"}
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return result


def run_long_prompt(impl: str, steps: int, gpus: int, prompt_tokens: int | None) -> dict:
    """Mistral-7B-architecture PRA model, batch 16: 128K-token prompts whose latest 4,096 tokens stay
    direct and the rest become implicit-head chunks, then greedy decode (tensor parallel)."""
    if impl == "reference":
        return _run_long_prompt_torch_arm(steps, gpus, prompt_tokens)
    rank, local, world = _env()
    torch.cuda.set_device(local)
    tp = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        from pdattention_b200.parallel.tp import TensorParallel

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        tp = TensorParallel()
    from pdattention_b200.inference.long_prompt import run_long_prompt_benchmark

    clocks = ClockSampler(local)
    out = run_long_prompt_benchmark(prompt_tokens=prompt_tokens or (1 << 17 if world > 1 else 1 << 15),
                                    new_tokens=max(steps, 16), tp=tp, clocks=clocks)
    result = {"metric": "PRA long-prompt decode tokens/s (Mistral-7B architecture, implicit head)",
              "value": out["decode_tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": out["decode_steps"],
              "warmup": 1, "ms_per_step": out["tpot_p50_ms"], "higher_is_better": True, "scaling": "strong",
              "vs_baseline": None, "dtype": "bf16",
              "data": "synthetic (uniform-random prompt token ids), random-init weights",
              "config": {k: out[k] for k in ("model", "batch", "prompt_tokens", "direct_window", "head_tokens",
                                             "new_tokens", "memory_gb_per_gpu", "position_offset")},
              "prefill_tokens_per_s": out["prefill_tokens_per_s"],
              "head_build_tokens_per_s": out["head_build_tokens_per_s"],
              "tail_prefill_tokens_per_s": out["tail_prefill_tokens_per_s"], "clocks": clocks.summary()}
    result["config"]["parallelism"] = f"tp{world}"
    if tp is not None:
        tp.close()
        import torch.distributed as dist

        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return result


def _run_long_prompt_torch_arm(steps: int, gpus: int, prompt_tokens: int | None) -> dict:
    """The long-prompt workload through ``baseline/torch_pra_decode.py`` (plain PyTorch + cuBLAS +
    NCCL; the reference itself has no Mistral-family model or tensor parallelism)."""
    rank, local, world = _env()
    if gpus != world:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    sys.path.insert(0, str(REPO / "baseline"))
    import torch_pra_decode

    clocks = ClockSampler(local)
    with clocks:
        out = torch_pra_decode.run_long_prompt(prompt_tokens=prompt_tokens or (1 << 17 if world > 1 else 1 << 15),
                                               new_tokens=max(steps, 16))
    result = {"metric": "PRA long-prompt decode tokens/s (Mistral-7B architecture, implicit head)",
              "value": out["decode_tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": out["decode_steps"],
              "warmup": 0, "ms_per_step": out["tpot_p50_ms"], "higher_is_better": True, "scaling": "strong",
              "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform-random prompt token ids), random-init weights",
              "config": {"model": "mistral-7b", "batch": out["batch"], "prompt_tokens": out["prompt_tokens"],
                         "direct_window": out["direct_window"], "head_tokens": out["head_tokens"],
                         "new_tokens": out["new_tokens"], "position_offset": out["position_offset"],
                         "parallelism": f"tp{world}"},
              "prefill_tokens_per_s": out["prefill_tokens_per_s"],
              "head_build_tokens_per_s": out["head_build_tokens_per_s"],
              "tail_prefill_tokens_per_s": out["tail_prefill_tokens_per_s"], "clocks": clocks.summary(),
              "gpu_launches": 0, "impl": "reference",
              "reference_kind": "the reference's prompt-overflow semantics in plain PyTorch + cuBLAS + NCCL "
                                "(baseline/torch_pra_decode.py); the reference itself has no Mistral-family or TP path"}
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return result


def run_memory_sweep(gpus: int, impl: str, steps: int, warmup: int):
    """Routing + memory-attention sweep of one Qwen2-7B-shaped PRA layer, memory sharded by chunk
    over the GPUs: 64K / 1M / 16M tokens x G in {1, 4} x chunk top-k in {4, 16, 64}.  One JSON
    line per configuration and arm (``fused``: this library's kernels and peer-memory
    collectives; ``baseline``: PyTorch operators and NCCL)."""
    rank, local, world = _env()
    if gpus != world:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    comm = group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        from pdattention_b200.parallel.tp import TensorParallel

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        comm = TensorParallel(max_partial_elems=1 << 10, max_gather_elems=4 << 20)
        group = dist.group.WORLD
    from pdattention_b200.inference.memory_sweep import run_sweep

    arms = ("baseline",) if impl == "reference" else ("fused", "baseline")
    for result in run_sweep(iters=max(steps, 5), warmup=warmup, comm=comm, group=group, arms=arms):
        result.update({"metric": "PRA layer routing + memory attention time (Qwen2-7B layer shapes)",
                       "unit": "us", "higher_is_better": False, "dtype": "bf16",
                       "data": "synthetic Gaussian K/V, chunk-sharded memory",
                       "baseline_note": "baseline = PyTorch operators + NCCL for the same math"})
        yield result
    if comm is not None:
        comm.close()
        import torch.distributed as dist

        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


class _Unavailable(RuntimeError):
    pass


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["pra", "reference"], default="pra")
    parser.add_argument("--workload", choices=["train", "decode", "memory-sweep", "long-prompt"], default="train",
                        help="train: TinyGPT-PRA data-parallel training (default); decode: PRA Llama-3-8B decode "
                             "with a chunk memory (tensor parallel over the GPUs)")
    parser.add_argument("--memory-tokens", type=int, default=None,
                        help="decode: total memory tokens (default 1M; 256K on one GPU, whose HBM cannot hold the "
                             "1M-token K/V of all 32 layers next to the weights and caches)")
    parser.add_argument("--batch", type=int, default=64)
    parser.add_argument("--reference-autocast", action="store_true",
                        help="train, --impl reference: run the reference's step under torch.autocast(bfloat16)")
    parser.add_argument("--prompt-tokens", type=int, default=None,
                        help="long-prompt: tokens per prompt (default 128K; 32K on one GPU)")
    args = parser.parse_args()
    rank = _env()[0]
    if args.workload == "long-prompt":
        result = run_long_prompt(args.impl, args.steps, args.gpus, args.prompt_tokens)
        if rank == 0:
            print(json.dumps(result))
        return
    if args.workload == "memory-sweep":
        for line in run_memory_sweep(args.gpus, args.impl, args.steps, max(args.warmup, 3)):
            if rank == 0:
                print(json.dumps(line), flush=True)
        return
    if args.workload == "decode":
        result = run_decode(args.impl, args.steps, max(args.warmup, 3), args.gpus, args.memory_tokens, args.batch)
        if rank == 0:
            print(json.dumps(result))
        return
    try:
        result = run(args.impl, args.steps, max(args.warmup, 3), args.gpus, args.reference_autocast)
    except _Unavailable as exc:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": str(exc)}))
        return
    if rank == 0:
        print(json.dumps(result))


if __name__ == "__main__":
    main()
