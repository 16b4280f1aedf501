"""Scalar metric helpers (``src/common/metrics.py``) plus device-side accumulation.

``grad_norm`` here computes the global norm with one fused reduction and one
host read (the reference reads one ``.item()`` per parameter).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import torch


@dataclass
class RunningAverages:
    totals: dict[str, float] = field(default_factory=dict)
    counts: dict[str, float] = field(default_factory=dict)

    def update(self, metrics: dict[str, float], weight: float = 1.0) -> None:
        w = float(weight)
        for key, value in metrics.items():
            self.totals[key] = self.totals.get(key, 0.0) + float(value) * w
            self.counts[key] = self.counts.get(key, 0.0) + w

    def compute(self) -> dict[str, float]:
        return {k: self.totals[k] / max(self.counts[k], 1) for k in self.totals}


def perplexity(loss: float) -> float:
    try:
        return float(math.exp(min(loss, 20.0)))
    except OverflowError:
        return float("inf")


def grad_norm(parameters) -> float:
    grads = [p.grad.detach() for p in parameters if p.grad is not None]
    if not grads:
        return 0.0
    norms = torch._foreach_norm(grads, 2.0)
    return float(torch.linalg.vector_norm(torch.stack([n.float() for n in norms]), 2.0).item())


def cuda_memory_allocated(device: str) -> float:
    if str(device).startswith("cuda") and torch.cuda.is_available():
        return float(torch.cuda.memory_allocated() / (1024 * 1024))
    return 0.0


class ThroughputTimer:
    def __init__(self):
        self.start = time.perf_counter()

    def rates(self, examples: int, tokens: int) -> dict[str, float]:
        elapsed = max(time.perf_counter() - self.start, 1e-9)
        return {"examples_per_second": examples / elapsed, "tokens_per_second": tokens / elapsed}


class DeviceTimer:
    """CUDA-event interval timer on the current stream (falls back to wall clock on CPU)."""

    def __init__(self, device: str):
        self.cuda = str(device).startswith("cuda") and torch.cuda.is_available()
        self._start = self._end = None
        self._t0 = 0.0

    def start(self) -> None:
        if self.cuda:
            self._start = torch.cuda.Event(enable_timing=True)
            self._end = torch.cuda.Event(enable_timing=True)
            self._start.record()
        else:
            self._t0 = time.perf_counter()

    def stop(self) -> None:
        if self.cuda:
            self._end.record()
        else:
            self._t0 = time.perf_counter() - self._t0

    def seconds(self) -> float:
        if self.cuda:
            self._end.synchronize()
            return self._start.elapsed_time(self._end) / 1000.0
        return self._t0
