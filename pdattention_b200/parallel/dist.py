"""Process-group bootstrap: one process per GPU, NCCL on CUDA, gloo on CPU.

Every multi-rank entry point reads ``RANK`` / ``LOCAL_RANK`` / ``WORLD_SIZE`` /
``MASTER_ADDR`` / ``MASTER_PORT`` from the environment (``torch.distributed.run``
sets them).  Process groups get a short timeout so ranks waiting on a peer
that died end with an error instead of hanging.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

DEFAULT_TIMEOUT_S = float(os.environ.get("PRA_PG_TIMEOUT_S", "120"))


def env_world() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def maybe_init_distributed(backend: str | None = None, timeout_s: float | None = None) -> tuple[int, int]:
    """Initialise the default group when launched with ``WORLD_SIZE > 1``; returns ``(rank, world)``.
    Rendezvous through ``MASTER_ADDR`` / ``MASTER_PORT``, or ``PRA_INIT_METHOD`` when set."""
    rank, local_rank, world = env_world()
    if world <= 1:
        return 0, 1
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    use_cuda = torch.cuda.is_available() and backend in (None, "nccl")
    if use_cuda:
        torch.cuda.set_device(local_rank)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kwargs = {"backend": backend or ("nccl" if use_cuda else "gloo"),
              "timeout": datetime.timedelta(seconds=timeout_s or DEFAULT_TIMEOUT_S), "rank": rank,
              "world_size": world}
    if use_cuda:
        kwargs["device_id"] = torch.device("cuda", local_rank)
    if os.environ.get("PRA_INIT_METHOD"):  # e.g. file:///path: a rendezvous that needs no TCP port
        kwargs["init_method"] = os.environ["PRA_INIT_METHOD"]
    dist.init_process_group(**kwargs)
    return rank, world


def world_info() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def barrier() -> None:
    if dist.is_available() and dist.is_initialized():
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a host scalar across ranks (device timings are reported as the max)."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    on_cuda = dist.get_backend() == "nccl"
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=(device or torch.device("cuda", torch.cuda.current_device())) if on_cuda else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def destroy() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
