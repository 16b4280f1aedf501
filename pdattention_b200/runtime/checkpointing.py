"""Checkpoint helpers (``src/common/checkpointing.py``).

Saves are atomic (temporary file then rename) so an interrupted save never
leaves a truncated ``latest.pt``; loading validates the payload and raises a
clear error for corrupt files, which is what restart-from-``latest.pt``
recovery relies on.
"""

from __future__ import annotations

import os
from dataclasses import asdict, is_dataclass
from pathlib import Path

import torch


class CheckpointError(RuntimeError):
    """A checkpoint file is missing, truncated or lacks required entries."""


def serializable_config(config) -> dict:
    if is_dataclass(config):
        return asdict(config)
    if hasattr(config, "__dict__"):
        return dict(config.__dict__)
    return dict(config)


def atomic_save(payload: dict, path) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    torch.save(payload, tmp)
    os.replace(tmp, path)
    return path


def read_checkpoint(path, map_location="cpu") -> dict:
    try:
        payload = torch.load(path, map_location=map_location, weights_only=False)
    except FileNotFoundError:
        raise
    except Exception as exc:  # truncated / corrupt archives
        raise CheckpointError(f"Checkpoint {path} could not be read: {exc}") from exc
    if not isinstance(payload, dict) or "model" not in payload:
        raise CheckpointError(f"Checkpoint {path} has no 'model' state.")
    return payload


def load_checkpoint(path, model, optimizer=None, scheduler=None, map_location="cpu") -> dict:
    checkpoint = read_checkpoint(path, map_location=map_location)
    model.load_state_dict(checkpoint["model"])
    if optimizer is not None and checkpoint.get("optimizer") is not None:
        optimizer.load_state_dict(checkpoint["optimizer"])
    if scheduler is not None and checkpoint.get("scheduler") is not None:
        scheduler.load_state_dict(checkpoint["scheduler"])
    return checkpoint
