"""Loop helpers: early stopping, checkpoint locations, learning-rate and progress readers.

Behaviour matches ``src/common/callbacks.py:7-57`` (patience counted in
validations without improvement; ``latest.pt`` / ``best.pt`` under one folder).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from pathlib import Path


@dataclass
class EarlyStopping:
    """``update(value)`` is True once ``patience`` consecutive values failed to beat the best
    (never, with ``patience=None``)."""

    patience: int | None
    best: float = math.inf
    bad_steps: int = 0

    def update(self, value: float) -> bool:
        if self.patience is None:
            return False
        improved = value < self.best
        self.best = value if improved else self.best
        self.bad_steps = 0 if improved else self.bad_steps + 1
        return not improved and self.bad_steps >= self.patience


class LearningRateMonitor:
    def current_lr(self, optimizer) -> float:
        """Learning rate of the optimizer's first parameter group."""
        return float(next(iter(optimizer.param_groups))["lr"])


class ProgressPrinter:
    def format(self, metrics: dict) -> str:
        """``key=value`` pairs (4 decimals) of the numeric entries."""
        return " ".join(f"{key}={value:.4f}" for key, value in metrics.items() if isinstance(value, (int, float)))


class ModelCheckpoint:
    """The run's checkpoint folder (created on construction) and its two file names."""

    LATEST, BEST = "latest.pt", "best.pt"

    def __init__(self, checkpoint_dir):
        self.checkpoint_dir = Path(checkpoint_dir)
        self.checkpoint_dir.mkdir(parents=True, exist_ok=True)

    latest_path = property(lambda self: self.checkpoint_dir / self.LATEST)
    best_path = property(lambda self: self.checkpoint_dir / self.BEST)
