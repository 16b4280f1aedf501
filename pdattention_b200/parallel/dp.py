"""Data-parallel gradient reduction for the device path.

Every rank holds the flat bf16 gradient buffer written by the backward GEMMs.
``GradientReducer.reduce`` turns it into the fp32 *average* gradient the fused
optimizer reads: NCCL all-reduce (sum) over an fp32 copy, with the 1/world
scale applied inside the optimizer kernel.  A fused peer-memory variant
(``pdattention_b200.parallel.peer``) replaces the NCCL call when symmetric
memory is available.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class GradientReducer:
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


def attach_data_parallel(model, optimizer, world_size: int) -> GradientReducer | None:
    """Route the fused optimizer through an all-reduced fp32 gradient (no-op for one rank)."""
    if world_size <= 1:
        return None
    runtime = model._device_runtime
    reducer = GradientReducer(runtime.flat, world_size)
    step = optimizer.step

    def reduced_step(closure=None):
        optimizer.grad_source = reducer.reduce()
        optimizer.grad_scale = 1.0 / world_size
        return step(closure)

    optimizer.step = reduced_step
    return reducer
