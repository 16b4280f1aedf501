"""Data-parallel gradient reduction for the device path.

Every rank holds the flat bf16 gradient buffer written by the backward GEMMs.
The reducer turns it into the fp32 *average* gradient the fused optimizer reads.

* ``PeerGradientReducer`` (the default on CUDA): the gradient buffer lives in
  symmetric memory and one kernel (``pra_ops.dp_allreduce``) reads every rank's
  bf16 slice over NVLink, sums in fp32, applies 1/world and stores the result
  into every rank's fp32 buffer -- cast, scale, reduce-scatter and all-gather
  fused, no staging copy and no NCCL call.
* ``NcclGradientReducer`` (the baseline, ``PRA_DP_BACKEND=nccl``): fp32 copy +
  NCCL all-reduce buckets, with the 1/world scale applied by the optimizer.

The reference has no data parallelism (one device in ``common/train.py``); the
gradient semantics are the reference's single-device AdamW on the batch mean,
so averaging over equally sized rank batches is the same update.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import _ext


class NcclGradientReducer:
    """fp32 copy of the flat gradient + NCCL all-reduce (sum) in buckets."""

    scale_in_optimizer = True

    def __init__(self, flat, world_size: int, bucket_elems: int = 64 << 20):
        self.flat = flat
        self.world = world_size
        self.bucket = bucket_elems
        self.buffer = torch.empty(flat.grad.numel(), device=flat.grad.device, dtype=torch.float32)

    def reduce(self) -> torch.Tensor:
        """fp32 sum of every rank's gradient (the caller scales by 1/world)."""
        self.buffer.copy_(self.flat.grad)
        if self.world > 1:
            for start in range(0, self.buffer.numel(), self.bucket):
                dist.all_reduce(self.buffer[start: start + self.bucket], op=dist.ReduceOp.SUM)
        return self.buffer

    def check(self) -> None:
        return None


GradientReducer = NcclGradientReducer  # backwards-compatible name


class PeerGradientReducer:
    """Fused peer-memory all-reduce of the flat gradient (one kernel per step)."""

    scale_in_optimizer = False

    def __init__(self, runtime, group=None, max_spins: int = 1 << 22):
        from .peer import PeerBuffers

        ext = _ext.require()
        flat = runtime.flat
        group = group or dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer reducer spans one NVLink domain of at most 8 GPUs")
        n = flat.grad.numel()
        self.numel = n
        self.buffers = PeerBuffers({"grad": (n, torch.bfloat16), "out": (n, torch.float32),
                                    "signals": (int(ext.dp_signal_words(self.world)), torch.int32)},
                                   group, flat.grad.device)
        self.src, self.dst, self.sig = (self.buffers.addresses(k) for k in ("grad", "out", "signals"))
        self.out = self.buffers.local("out")
        flat.rehome_grad(self.buffers.local("grad"), runtime.grad_views())
        self.epoch = 0
        self.max_spins = int(max_spins)
        self.error = torch.zeros(1, dtype=torch.int32, device=flat.grad.device)

    def reduce(self) -> torch.Tensor:
        """Average of every rank's gradient, in this rank's fp32 buffer."""
        self.epoch += 1
        _ext.require().dp_allreduce(self.src, self.dst, self.sig, self.rank, 0, self.numel, 1.0 / self.world,
                                    self.epoch, self.max_spins, self.error)
        return self.out

    def check(self) -> None:
        """Raise if any wait of a reduction timed out (a peer stopped or fell behind)."""
        code = int(self.error.item())
        if code:
            raise RuntimeError(f"peer gradient reduction: a wait timed out in phase {code - 1} "
                               "(a peer rank stopped or is not launching the reduction)")

    def close(self) -> None:
        self.buffers.close()


def _backend() -> str:
    return os.environ.get("PRA_DP_BACKEND", "peer").lower()


def attach_data_parallel(model, optimizer, world_size: int, backend: str | None = None):
    """Route the fused optimizer through the averaged gradient (no-op for one rank).

    ``backend``: ``"peer"`` (fused symmetric-memory kernel) or ``"nccl"``; default
    from ``PRA_DP_BACKEND`` (``peer``).
    """
    if world_size <= 1:
        return None
    runtime = model._device_runtime
    backend = (backend or _backend()).lower()
    if backend == "peer":
        reducer = PeerGradientReducer(runtime)
    elif backend == "nccl":
        reducer = NcclGradientReducer(runtime.flat, world_size)
    else:
        raise ValueError(f"unknown data-parallel backend {backend!r} (expected 'peer' or 'nccl')")
    step = optimizer.step

    def reduced_step(closure=None):
        optimizer.grad_source = reducer.reduce()
        optimizer.grad_scale = 1.0 / world_size if reducer.scale_in_optimizer else 1.0
        return step(closure)

    optimizer.step = reduced_step
    optimizer.reducer = reducer
    return reducer
