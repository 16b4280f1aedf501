"""Systems benchmarks of the reference's paper, measured through this framework.

Four measurements, each a list of CSV-ready rows with the reference's column
names where the quantity is the same:

* ``routing_speed`` (``scripts/run_pra_routing_speed.py``): per-example request
  latency and routing latency of the legacy scalar router, the tensorized router
  (both on the fp32 object path) and this framework's route kernel (device path),
  on fixed-target native-KV examples at split counts 32..256 for the ``tiny`` and
  ``small`` model tiers;
* ``routing_index_reuse`` (``scripts/run_pra_routing_index_reuse.py``): the
  routing index (the per-row chunk tables and gists) built once and reused
  (warm) against rebuilt per request (cold);
* ``kv_residency`` (``scripts/run_pra_kv_residency.py``): GPU-resident against
  CPU-resident K/V (pinned host pool, selected rows gathered over the host link),
  cold request (cache build + forward) and warm request (forward over a built
  cache), with the bytes that cross the link;
* ``batch_forward`` (``scripts/benchmark_batch_forward.py``): one prompt forward
  per row (the legacy singleton loop) against one batched forward.

Differences from the reference's protocol, by construction of this environment:
weights are random-initialised (the reference evaluates trained checkpoints;
latencies do not depend on the weights, losses do and are reported only as a
sanity value), the source is the synthetic fixed-position lookup with 255 facts
(HotpotQA / QASPER need corpora that are not on this machine), and references
are encoded independently (the device path's encoding strategy).  Times are
device times from CUDA events (routing) or synchronised wall clock around whole
requests (as the reference measures them).
"""

from __future__ import annotations

import copy
import random
import statistics
import string
import tempfile
import time
from pathlib import Path

import torch

from .config import PRAConfig, ResolverServiceConfig
from .data import PRADataModule, WordIdTokenizer
from .data.native_kv_benchmarks import EvidenceUnit, NativeKVBenchmarkExample, write_native_kv_benchmark

TIERS = {"tiny": dict(d_model=128, n_heads=4, n_layers=2, d_ff=256),
         "small": dict(d_model=256, n_heads=4, n_layers=4, d_ff=768)}
SPLITS = (32, 64, 128, 256)
STAGE = "synthetic_nativekv_fixed_target"
BACKENDS = ("legacy", "tensorized", "device")


def lookup_examples(n: int, units: int = 255, seed: int = 1729) -> list[NativeKVBenchmarkExample]:
    """``units`` one-bit facts ``<key>=<bit>`` per example (three-character keys), the queried
    fact first; the question names its key."""
    alphabet = string.ascii_lowercase + string.digits
    out = []
    for i in range(n):
        rng = random.Random(seed + 7919 * i)
        keys = set()
        while len(keys) < units:
            keys.add("".join(rng.choice(alphabet) for _ in range(3)))
        keys = sorted(keys)
        rng.shuffle(keys)
        bits = [str(rng.randrange(2)) for _ in keys]
        facts = tuple(EvidenceUnit(f"{k}={b}", j == 0) for j, (k, b) in enumerate(zip(keys, bits)))
        out.append(NativeKVBenchmarkExample(id=f"lookup-{i:05d}", source_units=facts, question=f"{keys[0]} =",
                                            answer=bits[0], metadata={"task_type": "fixed_position_lookup"}))
    return out


def _loader(root: Path, split: int, examples: int, tokenizer, batch_size: int = 1):
    write_native_kv_benchmark(root / f"split{split}", stage=STAGE, dataset_name="synthetic_native_kv",
                              split_count=split, examples=lookup_examples(examples),
                              generation_version="systems_lookup_v1")
    dm = PRADataModule(STAGE, str(root / f"split{split}"), batch_size=batch_size, max_seq_len=768,
                       tokenizer=tokenizer, shuffle=False).load()
    return [b for b in dm._loader(dm.dataset, shuffle=False)]


def _config(tier: str, vocab: int, backend: str, residency: str = "gpu") -> PRAConfig:
    return PRAConfig(vocab_size=vocab, max_seq_len=768, model_variant="td_pra", top_k_references=8,
                     top_k_chunks_per_reference=1, trigger_threshold=float("-inf"),
                     detail_materialization="selected_chunks", recursive_max_total_references=512,
                     recursive_max_total_tokens=65_536, kv_cache_residency=residency,
                     routing_backend="legacy" if backend == "legacy" else "tensorized",
                     collect_detailed_timing=backend != "device", device="cuda", **TIERS[tier])


def _model(cfg: PRAConfig, backend: str, seed: int = 0):
    from .models import TinyPRAModel
    from .models.fastpath import attach_device_runtime

    torch.manual_seed(seed)
    model = TinyPRAModel(copy.deepcopy(cfg)).cuda().eval()
    if backend == "device":
        attach_device_runtime(model)
        if model._device_runtime is None:
            raise RuntimeError("device path unavailable for the systems benchmark config")
        model._device_runtime.uniform_pra = False  # the per-layer path, whose routing launches are timed
        model._device_runtime.route_timer = []
    return model


def _request(model, batch, tokenizer):
    from .pra_train import _pra_batch_step

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.no_grad():
        loss, out = _pra_batch_step(model, batch, "cuda", tokenizer, ResolverServiceConfig(), None)
    torch.cuda.synchronize()
    return time.perf_counter() - t0, loss, out


def _routing_seconds(model, out) -> float:
    rt = getattr(model, "_device_runtime", None)
    if rt is not None and rt.route_timer is not None:
        torch.cuda.synchronize()
        total = sum(a.elapsed_time(b) for a, b in rt.route_timer) / 1000.0
        rt.route_timer.clear()
        return total
    return sum(float(d.get("routing_duration_seconds", 0.0)) for d in out["diagnostics"].values())


def _retrieved_tokens(model, out) -> float:
    rt = getattr(model, "_device_runtime", None)
    if rt is not None:
        return float(sum(int(r.ints[0].sum()) for r in rt.last_routing.values()))
    return float(sum(d.get("memory_tokens_materialized", 0.0) for d in out["diagnostics"].values()))


def routing_speed(tiers=("tiny", "small"), splits=SPLITS, examples: int = 32, backends=BACKENDS,
                  root: Path | None = None) -> list[dict]:
    """Per-example request and routing latency of each router (batch 1, after one warm-up example)."""
    root = Path(root or tempfile.mkdtemp(prefix="pra_systems_"))
    tokenizer = WordIdTokenizer(8000)
    rows = []
    for tier in tiers:
        for split in splits:
            batches = _loader(root, split, examples + 1, tokenizer)
            legacy_route = None
            for backend in backends:
                model = _model(_config(tier, tokenizer.vocab_size, backend), backend)
                _request(model, batches[0], tokenizer)  # warm-up (kernel set-up, allocator)
                _routing_seconds(model, {"diagnostics": {}})
                lat, route, losses, tokens = [], [], [], []
                for batch in batches[1:]:
                    seconds, loss, out = _request(model, batch, tokenizer)
                    lat.append(seconds)
                    route.append(_routing_seconds(model, out))
                    losses.append(float(loss))
                    tokens.append(_retrieved_tokens(model, out))
                routing = statistics.fmean(route)
                if backend == "legacy":
                    legacy_route = routing
                rows.append({"model_tier": tier, "split_count": split, "routing_backend": backend,
                             "examples": len(lat), "loss": statistics.fmean(losses),
                             "request_latency_seconds": statistics.fmean(lat),
                             "routing_latency_seconds": routing,
                             "gist_comparisons": (split - 1) * TIERS[tier]["n_layers"],
                             "retrieved_physical_kv_tokens": statistics.fmean(tokens),
                             "routing_speedup_vs_legacy": (legacy_route / routing) if legacy_route and routing else None})
    return rows


def kv_residency(tiers=("tiny", "small"), splits=(32, 64, 128, 256), examples: int = 16, warm_repeats: int = 8,
                 root: Path | None = None) -> list[dict]:
    """GPU- against CPU-resident K/V on the device path: cold request (build + forward), warm
    request (``warm_repeats`` forwards over the built cache), bytes the selected rows move."""
    root = Path(root or tempfile.mkdtemp(prefix="pra_systems_"))
    tokenizer = WordIdTokenizer(8000)
    rows = []
    for tier in tiers:
        d, layers = TIERS[tier]["d_model"], TIERS[tier]["n_layers"]
        for split in splits:
            batches = _loader(root, split, examples + 1, tokenizer)
            for residency in ("gpu", "cpu"):
                model = _model(_config(tier, tokenizer.vocab_size, "device", residency), "device")
                rt = model._device_runtime
                rt.uniform_pra, rt.route_timer = True, None  # the native stacks (timing is wall clock)
                _request(model, batches[0], tokenizer)
                cold, warm, moved, cached, on_gpu = [], [], [], [], []
                for batch in batches[1:]:
                    seconds, _, out = _request(model, batch, tokenizer)
                    cold.append(seconds)
                    memory = out["memory"]
                    ids = batch["input_ids"].cuda()
                    mask = batch["attention_mask"].cuda()
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                    with torch.no_grad():
                        for _ in range(warm_repeats):
                            rt.prompt_forward(ids, mask, memory)
                    torch.cuda.synchronize()
                    warm.append((time.perf_counter() - t0) / warm_repeats)
                    selected = sum(int(r.ints[0].sum()) for r in rt.last_routing.values())
                    moved.append(selected * 2 * d * 2 if residency == "cpu" else 0)
                    cached.append(out["metrics"]["cached_kv_bytes"])
                    on_gpu.append(out["metrics"]["gpu_cached_kv_bytes"])
                rows.append({"model_tier": tier, "split_count": split, "kv_cache_residency": residency,
                             "examples": len(cold), "cached_kv_bytes": statistics.fmean(cached),
                             "gpu_cached_kv_bytes": statistics.fmean(on_gpu),
                             "selected_kv_transfer_bytes": statistics.fmean(moved),
                             "cold_request_ms": 1000 * statistics.fmean(cold),
                             "warm_request_ms": 1000 * statistics.fmean(warm), "layers": layers})
    return rows


def routing_index_reuse(tiers=("tiny", "small"), splits=SPLITS, examples: int = 16, root: Path | None = None):
    """Cold (routing index built with the request: cache build + forward) against warm (index
    reused: forward over an already built memory) on the device path, with the index's bytes."""
    root = Path(root or tempfile.mkdtemp(prefix="pra_systems_"))
    tokenizer = WordIdTokenizer(8000)
    rows = []
    for tier in tiers:
        for split in splits:
            batches = _loader(root, split, examples + 1, tokenizer)
            model = _model(_config(tier, tokenizer.vocab_size, "device"), "device")
            rt = model._device_runtime
            _request(model, batches[0], tokenizer)
            _routing_seconds(model, {"diagnostics": {}})
            cold, warm, route, index = [], [], [], []
            for batch in batches[1:]:
                seconds, _, out = _request(model, batch, tokenizer)
                cold.append(seconds)
                _routing_seconds(model, out)
                memory = out["memory"]
                ids, mask = batch["input_ids"].cuda(), batch["attention_mask"].cuda()
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                with torch.no_grad():
                    rt.prompt_forward(ids, mask, memory)
                torch.cuda.synchronize()
                warm.append(time.perf_counter() - t0)
                route.append(_routing_seconds(model, out))
                index.append(memory.gist_tables.numel() * 4 + memory.gist_count_all.numel() * 4)
            rows.append({"model_tier": tier, "split_count": split, "examples": len(cold),
                         "candidate_chunks": split - 1, "index_bytes": statistics.fmean(index),
                         "tensorized_cold_index_ms": 1000 * statistics.fmean(cold),
                         "tensorized_warm_index_ms": 1000 * statistics.fmean(warm),
                         "query_scoring_ms": 1000 * statistics.fmean(route),
                         "warm_speedup": statistics.fmean(cold) / max(statistics.fmean(warm), 1e-12)})
    return rows


def batch_forward(batch_sizes=(1, 2, 4, 8, 32), repeats: int = 3, tier: str = "small", split: int = 32,
                  root: Path | None = None) -> list[dict]:
    """One prompt forward per row (the legacy singleton loop) against one batched forward over
    the same built memory (device path)."""
    root = Path(root or tempfile.mkdtemp(prefix="pra_systems_"))
    tokenizer = WordIdTokenizer(8000)
    rows = []
    for bs in batch_sizes:
        (batch,) = _loader(root / f"b{bs}", split, bs, tokenizer, batch_size=bs)[:1]
        model = _model(_config(tier, tokenizer.vocab_size, "device"), "device")
        rt = model._device_runtime
        rt.uniform_pra, rt.route_timer = True, None
        _, _, out = _request(model, batch, tokenizer)
        memory = out["memory"]
        ids, mask = batch["input_ids"].cuda(), batch["attention_mask"].cuda()

        def timed(fn):
            fn()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(repeats):
                fn()
            torch.cuda.synchronize()
            return (time.perf_counter() - t0) / repeats

        with torch.no_grad():
            batched = timed(lambda: rt.prompt_forward(ids, mask, memory))
            # singleton: each row alone against its own memory (its own cache build, as the loop runs it)
            singles = []
            for r in range(bs):
                one = {k: (v[r: r + 1] if torch.is_tensor(v) else [v[r]] if isinstance(v, list) else v)
                       for k, v in batch.items()}
                _, _, o1 = _request(model, one, tokenizer)
                singles.append((one["input_ids"].cuda(), one["attention_mask"].cuda(), o1["memory"]))
            single = timed(lambda: [rt.prompt_forward(i, m, mem) for i, m, mem in singles])
        tokens = int(batch["attention_mask"].sum())
        rows.append({"batch_size": bs, "tokens": tokens, "legacy_prompt_forward_calls": bs,
                     "batched_prompt_forward_calls": 1, "legacy_prompt_seconds": single,
                     "batched_prompt_seconds": batched, "speedup": single / max(batched, 1e-12),
                     "batched_examples_per_second": bs / batched, "batched_tokens_per_second": tokens / batched})
    return rows


SUITES = {"routing-speed": routing_speed, "routing-index-reuse": routing_index_reuse, "kv-residency": kv_residency,
          "batch-forward": batch_forward}


def main(argv=None) -> None:
    import argparse
    import csv
    import json
    import sys

    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("suite", choices=sorted(SUITES))
    parser.add_argument("--csv", default=None, help="also write the rows to this CSV file")
    parser.add_argument("--quick", action="store_true", help="tiny tier, split counts 32 and 256, 8 examples")
    args = parser.parse_args(argv)
    torch.cuda.set_device(0)
    kwargs = {}
    if args.quick and args.suite != "batch-forward":
        kwargs = dict(tiers=("tiny",), splits=(32, 256), examples=8)
    rows = SUITES[args.suite](**kwargs)
    for row in rows:
        print(json.dumps(row))
    if args.csv:
        with open(args.csv, "w", newline="") as fh:
            writer = csv.DictWriter(fh, fieldnames=list(rows[0]))
            writer.writeheader()
            writer.writerows(rows)
    sys.stdout.flush()


if __name__ == "__main__":
    main()
