"""Experiment logging: one metrics sink fanning out to pluggable backends.

The reference exposes one logger class per tracker (``src/common/logging.py:10-171``:
console, TensorBoard, W&B, ClearML, a multiplexer and ``build_logger``).  Here a
``MetricsSink`` owns the fan-out and does the work every tracker shares once per
call (keeping the numeric values, naming scalars ``split/key``); a backend only
says where a scalar, a text or the run configuration goes.  Optional trackers
that cannot be imported or initialised become no-op backends, so a missing
package never stops a run.  Under data parallelism only rank 0 gets real
backends (``build_logger(..., rank=r)``).

The class names of the reference (``ConsoleLogger``, ``TensorBoardLogger``,
``WandBLogger``, ``ClearMLLogger``, ``MultiLogger``) remain importable: each is
a backend (or the sink) with the constructor signature users know.
"""

from __future__ import annotations

from pathlib import Path

from .plots import MetricsHistory


def _scalars(metrics: dict) -> dict[str, float]:
    return {k: v for k, v in metrics.items() if isinstance(v, (int, float))}


class ExperimentLogger:
    """The logging interface every backend and the sink implement (all methods optional)."""

    def log_metrics(self, metrics: dict, step: int, split: str) -> None:
        pass

    def log_text(self, name: str, text: str, step: int) -> None:
        pass

    def log_config(self, config) -> None:
        pass

    def close(self) -> None:
        pass


class _Backend(ExperimentLogger):
    """A destination for already-filtered scalars; subclasses override ``scalars``."""

    def scalars(self, values: dict[str, float], step: int, split: str) -> None:
        pass

    def log_metrics(self, metrics: dict, step: int, split: str) -> None:
        self.scalars(_scalars(metrics), step, split)


class ConsoleLogger(_Backend):
    """``[split step=N] key=value ...`` lines on stdout."""

    def scalars(self, values, step, split):
        print(f"[{split} step={step}] " + " ".join(f"{k}={v:.4f}" for k, v in values.items()))

    def log_text(self, name, text, step):
        print(f"[text step={step}] {name}: {text}")

    def log_config(self, config):
        print(f"[config] {config}")


class TensorBoardLogger(_Backend):
    """TensorBoard event files under ``log_dir``; without ``tensorboard`` installed, a
    tab-separated ``events.out.tfevents.fallback`` file receives the same records."""

    def __init__(self, log_dir):
        self.log_dir = Path(log_dir)
        self.log_dir.mkdir(parents=True, exist_ok=True)
        self.fallback_path = self.log_dir / "events.out.tfevents.fallback"
        try:
            from torch.utils.tensorboard import SummaryWriter

            self.writer = SummaryWriter(str(self.log_dir))
        except Exception:  # tensorboard missing or unusable
            self.writer = None
            self.fallback_path.touch()

    def log_metrics(self, metrics, step, split):
        if self.writer is None:
            with self.fallback_path.open("a", encoding="utf-8") as out:
                out.write(f"{step}\t{split}\t{metrics}\n")
        else:
            super().log_metrics(metrics, step, split)

    def scalars(self, values, step, split):
        for key, value in values.items():
            self.writer.add_scalar(f"{split}/{key}", value, step)

    def log_text(self, name, text, step):
        if self.writer is not None:
            self.writer.add_text(name, text, step)

    def log_config(self, config):
        self.log_text("config", str(config), 0)

    def close(self):
        if self.writer is not None:
            self.writer.close()


class _HostedTracker(_Backend):
    """A hosted tracker opened with ``open(config)``; any failure leaves it disabled."""

    def __init__(self, config, enabled: bool):
        self.handle = None
        if enabled:
            try:
                self.handle = self.open(config)
            except Exception:  # package missing, offline, bad credentials
                self.handle = None

    def open(self, config):
        raise NotImplementedError

    def log_metrics(self, metrics, step, split):
        if self.handle is not None:
            self.publish(metrics, step, split)

    def publish(self, metrics, step, split):
        self.scalars(_scalars(metrics), step, split)


class WandBLogger(_HostedTracker):
    def open(self, config):
        import wandb

        return wandb.init(project=config.wandb_project, config=dict(config.__dict__),
                          name=getattr(config, "experiment_name", None))

    def publish(self, metrics, step, split):
        self.handle.log({f"{split}/{k}": v for k, v in metrics.items()}, step=step)

    def close(self):
        if self.handle is not None:
            self.handle.finish()


class ClearMLLogger(_HostedTracker):
    def open(self, config):
        from clearml import Task

        task = Task.init(project_name=config.clearml_project, task_name=getattr(config, "experiment_name", "experiment"))
        task.connect(dict(config.__dict__))
        return task

    def scalars(self, values, step, split):
        report = self.handle.get_logger().report_scalar
        for key, value in values.items():
            report(split, key, value, iteration=step)


class MetricsSink(ExperimentLogger):
    """Forwards every call to each backend in order."""

    def __init__(self, backends: list[ExperimentLogger]):
        self.loggers = list(backends)

    def _each(self, method: str, *args) -> None:
        for backend in self.loggers:
            getattr(backend, method)(*args)

    def log_metrics(self, metrics, step, split):
        self._each("log_metrics", metrics, step, split)

    def log_text(self, name, text, step):
        self._each("log_text", name, text, step)

    def log_config(self, config):
        self._each("log_config", config)

    def close(self):
        self._each("close")


MultiLogger = MetricsSink


# Optional trackers keyed by the TrainConfig switch that enables them.
_TRACKERS = (("use_wandb", WandBLogger), ("use_clearml", ClearMLLogger))


def build_logger(config, run_dir, *, rank: int = 0) -> ExperimentLogger:
    """The run's sink: console + metric history (+ TensorBoard and hosted trackers when enabled);
    a no-op logger on ranks other than 0."""
    if rank != 0:
        return ExperimentLogger()
    backends: list[ExperimentLogger] = [
        ConsoleLogger(), MetricsHistory(run_dir, save_plots=getattr(config, "save_metric_plots", True))]
    if getattr(config, "use_tensorboard", False):
        backends.append(TensorBoardLogger(Path(run_dir) / "tensorboard"))
    backends += [cls(config, bool(getattr(config, flag, False))) for flag, cls in _TRACKERS]
    return MetricsSink(backends)
