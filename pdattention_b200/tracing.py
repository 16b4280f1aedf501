"""NVTX ranges around the framework's phases (visible in Nsight Systems / Nsight Compute).

The reference times its phases on the host (``collect_detailed_timing``:
synchronise, read the clock; ``src/pra_torch/attention.py:21-24,377-419``).
The device path never synchronises inside a step, so it marks its phases with
NVTX ranges instead: a profiler attached to the process shows the cache build,
routing, the block stack (one range per layer, pushed by the C++ executor), the
loss, the backward and the optimizer on its timeline, and ``ncu --nvtx
--nvtx-include`` can select the kernels of one phase.  With no tool attached a
range costs one call into NVTX's no-op stub.  ``PRA_NVTX=0`` turns the Python
ranges off.
"""

from __future__ import annotations

import contextlib
import functools
import os

import torch

ENABLED = os.environ.get("PRA_NVTX", "1") != "0"


@contextlib.contextmanager
def nvtx_range(name: str):
    """Mark ``name`` on the NVTX timeline for the duration of the ``with`` body."""
    if not ENABLED or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def traced(name: str):
    """Decorator form of ``nvtx_range``."""

    def wrap(fn):
        @functools.wraps(fn)
        def inner(*args, **kwargs):
            with nvtx_range(name):
                return fn(*args, **kwargs)

        return inner

    return wrap
