"""Shared fixtures.

``ref`` imports the reference implementation (the CPU oracle) from the
``baseline/_ref`` install when present, else from a source checkout named by
``PRA_REFERENCE_SRC``; tests that need it are skipped when neither exists.
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running")


def _reference_root() -> Path | None:
    installed = REPO / "baseline" / "_ref"
    if (installed / "pra_torch").exists():
        return installed
    src = os.environ.get("PRA_REFERENCE_SRC")
    if src and (Path(src) / "pra_torch").exists():
        return Path(src)
    return None


@pytest.fixture(scope="session")
def ref():
    root = _reference_root()
    if root is None:
        pytest.skip("reference implementation not installed")
    sys.dont_write_bytecode = True
    if str(root) not in sys.path:
        sys.path.append(str(root))
    names = ["pra_torch.config", "pra_torch.model", "pra_torch.memory", "pra_torch.chunking", "pra_torch.gists",
             "pra_torch.cache_services", "pra_torch.prompt", "pra_torch.resolution", "pra_torch.memory_batching",
             "data.collators", "data.tokenizer", "data.datamodules", "pra_core.references", "common.metrics",
             "pra_torch.metrics", "pra_torch.native_metrics", "common.recall_sparsity"]
    mods = {n.split(".")[-1] if n != "data.tokenizer" else "tokenizer": importlib.import_module(n) for n in names}
    return SimpleNamespace(**mods)


@pytest.fixture
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
