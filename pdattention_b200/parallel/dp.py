"""Data-parallel gradient reduction for the device path.

Every rank holds the flat bf16 gradient buffer written by the backward GEMMs.
The reducer turns it into the fp32 *average* gradient the fused optimizer reads.

* ``PeerGradientReducer`` (the default on CUDA): the gradient buffer lives in
  symmetric memory and a kernel (``pra_ops.dp_allreduce``) reads every rank's
  bf16 slice over NVLink, sums in fp32 (ranks in a fixed order), applies 1/world
  and stores the average into every rank's buffer -- cast, scale,
  reduce-scatter and all-gather fused, no staging copy and no NCCL call.  By
  default the average is stored as bf16 back into the gradient buffers (2 bytes
  per element and peer cross NVLink, as many as the gradients themselves);
  ``PRA_DP_OUT=fp32`` stores an fp32 average into a separate buffer instead.
  With ``PRA_DP_OVERLAP=1`` the reduction overlaps the backward: each block's
  gradient range is reduced on a side stream as soon as the block's backward has
  written it.
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


def reduction_ranges(flat) -> tuple[list[tuple[int, int]], tuple[int, int]]:
    """(per-layer (start, count) element ranges of the flat gradient, the LM head's range): each
    block's parameters are contiguous in the flat layout, and so is the head (last, with its
    padding rows)."""
    offsets = flat.offsets
    layers = []
    i = 0
    while f"blocks.{i}.attn.q_proj.weight" in offsets:
        start = offsets[f"blocks.{i}.attn.q_proj.weight"]
        end = offsets.get(f"blocks.{i + 1}.attn.q_proj.weight", offsets["token_emb.weight"])
        layers.append((start, end - start))
        i += 1
    head = offsets["head.weight"]
    return layers, (head, flat.total - head)


class PeerGradientReducer:
    """Fused peer-memory all-reduce of the flat gradient.

    With ``overlap`` (``PRA_DP_OVERLAP=1``; off by default) the reduction is launched
    in pieces during the backward on a communication stream: the LM head's gradient as soon as
    the block stack's backward starts, and each block's gradient as soon as that block's
    backward has written it (hooks called by the native training stack); the embeddings and
    final norm, finished last, are reduced when the optimizer asks.  The overlapped launches
    use ``overlap_blocks`` CTAs so the backward keeps most SMs.  Every rank launches the same
    pieces in the same order.
    """

    scale_in_optimizer = False

    def __init__(self, runtime, group=None, max_spins: int = 1 << 22, overlap: bool | None = None,
                 overlap_blocks: int = 64, out_dtype: str | None = None):
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
        out_dtype = (out_dtype or os.environ.get("PRA_DP_OUT", "bf16")).lower()
        if out_dtype not in ("bf16", "fp32"):
            raise ValueError(f"PRA_DP_OUT must be bf16 or fp32, not {out_dtype!r}")
        self.in_place = out_dtype == "bf16"
        spec = {"grad": (n, torch.bfloat16), "signals": (int(ext.dp_signal_words(self.world)), torch.int32)}
        if not self.in_place:
            spec["out"] = (n, torch.float32)
        self.buffers = PeerBuffers(spec, group, flat.grad.device)
        self.src, self.sig = self.buffers.addresses("grad"), self.buffers.addresses("signals")
        self.dst = [] if self.in_place else self.buffers.addresses("out")  # [] = in place, bf16
        flat.rehome_grad(self.buffers.local("grad"), runtime.grad_views())
        self.out = self.buffers.local("grad") if self.in_place else self.buffers.local("out")
        self.epoch = 0
        self.max_spins = int(max_spins)
        self.error = torch.zeros(1, dtype=torch.int32, device=flat.grad.device)
        if overlap is None:
            overlap = os.environ.get("PRA_DP_OVERLAP", "0") != "0"
        self.overlap = bool(overlap) and self.world > 1
        self.overlap_blocks = int(overlap_blocks)
        self.layer_ranges, self.head_range = reduction_ranges(flat)
        self.done: list[tuple[int, int]] = []  # ranges already launched this step
        self.comm = torch.cuda.Stream(device=flat.grad.device) if self.overlap else None
        if self.overlap:
            runtime.grad_hooks = self

    def _launch(self, start: int, count: int, blocks: int = 0) -> None:
        self.epoch += 1
        _ext.require().dp_allreduce(self.src, self.dst, self.sig, self.rank, start, count, 1.0 / self.world,
                                    self.epoch, self.max_spins, self.error, blocks)

    def _launch_async(self, rng: tuple[int, int]) -> None:
        ready = torch.cuda.Event()
        ready.record()  # after the kernels that wrote this range (current stream)
        self.comm.wait_event(ready)
        with torch.cuda.stream(self.comm):
            self._launch(rng[0], rng[1], self.overlap_blocks)
        self.done.append(rng)

    # hooks called by the native training stack's backward
    def before_stack(self) -> None:
        self._launch_async(self.head_range)

    def after_layer(self, layer: int) -> None:
        self._launch_async(self.layer_ranges[layer])

    def reduce(self) -> torch.Tensor:
        """Average of every rank's gradient, in this rank's fp32 buffer (ordered before the
        caller's next kernels on the current stream)."""
        if not self.done:
            self._launch(0, self.numel)
            return self.out
        rest, cursor = [], 0
        for start, count in sorted(self.done):
            if start > cursor:
                rest.append((cursor, start - cursor))
            cursor = max(cursor, start + count)
        if cursor < self.numel:
            rest.append((cursor, self.numel - cursor))
        ready = torch.cuda.Event()
        ready.record()
        self.comm.wait_event(ready)
        with torch.cuda.stream(self.comm):
            for start, count in rest:
                self._launch(start, count)
        torch.cuda.current_stream().wait_stream(self.comm)
        self.done = []
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


def attach_data_parallel(model, optimizer, world_size: int, backend: str | None = None,
                         overlap: bool | None = None, out_dtype: str | None = None):
    """Route the fused optimizer through the averaged gradient (no-op for one rank).

    ``backend``: ``"peer"`` (fused symmetric-memory kernel) or ``"nccl"``; default
    from ``PRA_DP_BACKEND`` (``peer``).  ``out_dtype`` (peer backend): ``"bf16"`` (average
    written back in place, the default) or ``"fp32"`` (separate fp32 buffer).
    """
    if world_size <= 1:
        return None
    runtime = model._device_runtime
    backend = (backend or _backend()).lower()
    if backend == "peer":
        reducer = PeerGradientReducer(runtime, overlap=overlap, out_dtype=out_dtype)
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
