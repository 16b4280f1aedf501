"""Device-time benchmarks of the fused compute + collective kernels, with their rooflines.

Run one process per GPU (``torchrun --nproc-per-node N -m pdattention_b200.collective_bench``);
every timing is CUDA events on the launching stream around ``iters`` launches after
warm-up, the max over ranks.  The roofline of a fused kernel is the slower of its compute
(or HBM traffic) at the measured peak and the bytes that must cross NVLink at the
measured peer-copy rate (770 GB/s per direction per GPU on this pool):

* ``dp_allreduce``: the data-parallel gradient reduction of the TinyGPT-PRA-163M flat
  buffer (bf16 in place).  Rank r reduces slice r: it reads that slice from its w-1 peers
  while they read their slices from it, then stores its result into every peer while they
  store theirs into it, so each link direction carries 2 (w-1)/w of the buffer (the
  all-reduce "bus" volume);
* ``decode_gemm_allreduce``: the row-parallel decode projections (64 rows; Llama-3-8B O
  and down shards) with the partial pushed to every rank and summed where it lands,
  against the unfused GEMM + one-shot all-reduce; HBM floor = the weight shard read once;
* ``route_exchange``: local top-k with the cross-GPU candidate exchange and merge fused
  in, against local top-k + all-gather + merge.
"""

from __future__ import annotations

import datetime
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU


def _peaks() -> dict:
    from pathlib import Path

    path = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    try:
        return json.loads(path.read_text())
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def _time(fn, iters: int, world: int, device) -> float:
    """Mean device microseconds per call, max over ranks."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier(device_ids=[device.index])
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    us = torch.tensor([1000.0 * s.elapsed_time(e) / iters], dtype=torch.float64, device=device)
    dist.all_reduce(us, op=dist.ReduceOp.MAX)
    return float(us.item())


def dp_allreduce(world: int, rank: int, device, iters: int = 20, numel: int = 163_000_000) -> dict:
    from .ops import _ext
    from .parallel.peer import PeerBuffers

    ext = _ext.require()
    n = numel // 8 * 8
    bufs = PeerBuffers({"grad": (n, torch.bfloat16), "sig": (int(ext.dp_signal_words(world)), torch.int32)},
                       device=device)
    grad = bufs.local("grad")
    grad.normal_()
    src, sig = bufs.addresses("grad"), bufs.addresses("sig")
    error = torch.zeros(1, dtype=torch.int32, device=device)
    state = {"epoch": 0}

    def call():
        state["epoch"] += 1
        ext.dp_allreduce(src, [], sig, rank, 0, n, 1.0 / world, state["epoch"], 1 << 22, error, 0)

    us = _time(call, iters, world, device)
    assert int(error.item()) == 0, "a wait of the reduction timed out"
    link_bytes = 2 * (world - 1) / world * 2 * n  # per direction per GPU: peer reads + result stores, bf16
    floor_us = link_bytes / (NVLINK_GBS * 1e3)
    bufs.close()
    return {"case": "dp_allreduce (bf16 in place)", "elements": n, "us": us,
            "nvlink_gb_per_direction": link_bytes / 1e9, "bus_gbs": link_bytes / us / 1e3,
            "roofline_us": floor_us, "fraction_of_roofline": floor_us / us}


def decode_gemm_allreduce(world: int, rank: int, device, iters: int = 50) -> list[dict]:
    from .parallel.tp import TensorParallel

    peaks = _peaks()
    tp = TensorParallel()
    gen = torch.Generator(device=device).manual_seed(rank)
    rows = []
    for name, n, k in (("o_proj", 4096, 4096 // world), ("down_proj", 4096, 14336 // world)):
        x = torch.randn(64, k, device=device, generator=gen).bfloat16()
        w = (torch.randn(n, k, device=device, generator=gen) * 0.02).bfloat16()
        res = torch.randn(64, n, device=device, generator=gen).bfloat16()
        fused = _time(lambda: tp.fused_gemm_allreduce(x, w, res), iters, world, device)
        unfused = _time(lambda: tp.gemm_allreduce(x, w, res), iters, world, device)
        hbm_bytes = n * k * 2 + 64 * k * 2 + 2 * 64 * n * 2
        link_bytes = (world - 1) * 64 * n * 2
        floor_us = max(hbm_bytes / (peaks["hbm_gbs"] * 1e3), link_bytes / (NVLINK_GBS * 1e3),
                       2 * 64 * n * k / (peaks["bf16_tflops"] * 1e6))
        rows.append({"case": f"decode {name} GEMM + all-reduce, 64 rows, weight shard {n}x{k}", "fused_us": fused,
                     "gemm_then_allreduce_us": unfused, "roofline_us": floor_us,
                     "fraction_of_roofline": floor_us / fused, "hbm_mb": hbm_bytes / 1e6,
                     "nvlink_kb_per_direction": link_bytes / 1e3})
    tp.check()
    tp.close()
    return rows


def route_exchange(world: int, rank: int, device, iters: int = 50, chunks: int = 16384, width: int = 1024,
                   k: int = 16) -> dict:
    import torch.nn.functional as F

    from .ops import _ext
    from .parallel.tp import TensorParallel

    ext = _ext.require()
    tp = TensorParallel()
    gen = torch.Generator(device=device).manual_seed(5)  # identical on every rank
    gists = F.normalize(torch.randn(chunks, width, device=device, generator=gen), dim=-1)
    query = torch.randn(64, width, device=device, generator=gen)
    per = chunks // world
    c0 = rank * per
    local = gists[c0: c0 + per].contiguous()
    scores = (F.normalize(query, dim=-1) @ local.t()).contiguous()
    lo = torch.zeros(64, dtype=torch.int32, device=device)
    hi = torch.full((64,), per, dtype=torch.int32, device=device)
    clen = torch.full((chunks,), 64, dtype=torch.int32, device=device)
    row0 = torch.arange(chunks, dtype=torch.int32, device=device) * 64
    mem_max = k * 64

    def fused():
        tp.route_exchange(scores, query, local, lo, hi, k, 4 * k, -1, mem_max, c0, 1, clen, row0)

    def unfused():
        cs, ci = ext.route_topk(scores, query, local, lo, hi, clen, row0, k, 4 * k, -1, 0, True, c0, 1, 1)
        merged = tp.all_gather_columns(torch.cat([cs, ci.view(torch.float32)], dim=1))
        ext.route_merge(merged, world, k, -1, clen, row0, mem_max, False)

    out = {"case": f"routing top-{k} over {chunks} chunks ({per} per rank), 64 rows: local top-k + exchange + merge",
           "fused_us": _time(fused, iters, world, device), "topk_allgather_merge_us": _time(unfused, iters, world, device)}
    tp.check()
    tp.close()
    return out


def main() -> None:
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    world, rank = dist.get_world_size(), dist.get_rank()
    results = [dp_allreduce(world, rank, device)]
    results += decode_gemm_allreduce(world, rank, device)
    results.append(route_exchange(world, rank, device))
    if rank == 0:
        for r in results:
            print(json.dumps({"world": world, **r}))
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
