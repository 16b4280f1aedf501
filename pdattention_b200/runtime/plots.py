"""Metric history of a run and the files written from it.

Outputs (the reference's layout, ``src/common/plots.py:29-168``, so existing
tooling reads them): ``metrics.json`` = ``{"config": ..., "records": [...]}``
with one record per logged call (``step``, ``split``, the loop counters such as
``epoch`` / ``batch_step`` lifted out of the metrics, and ``metrics``: the other
scalar values); ``metrics.md`` with the latest record of each split and links to
the plots; ``plots/<metric>.png`` drawn headless (Agg), one line per split, or
``plots/plotting_unavailable.txt`` when matplotlib cannot be imported.
"""

from __future__ import annotations

import itertools
import json
from dataclasses import asdict, is_dataclass
from pathlib import Path

# Loop counters that describe WHERE a record was taken rather than what was measured.
_RECORD_DIMENSIONS = frozenset({"epoch", "batch_in_epoch", "batch_step", "optimizer_step", "optimizer_updated",
                                "batches"})


def _jsonable_config(config):
    """The configuration as JSON-ready data (a dict when it has fields, else its string)."""
    if is_dataclass(config) and not isinstance(config, type):
        return asdict(config)
    if isinstance(config, dict):
        return dict(config)
    return dict(vars(config)) if hasattr(config, "__dict__") else str(config)


def make_record(metrics: dict, step: int, split: str) -> dict | None:
    """One history record, or ``None`` when ``metrics`` holds no measured scalar."""
    measured, where = {}, {}
    for key, value in metrics.items():
        if isinstance(value, (int, float)):
            (where if key in _RECORD_DIMENSIONS else measured)[key] = float(value)
    if not measured:
        return None
    return {"step": int(step), "split": str(split), **where, "metrics": measured}


def save_metrics_json(path, records: list[dict], config=None) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps({"config": _jsonable_config(config), "records": records}, indent=2, default=str),
                    encoding="utf-8")
    return path


def _markdown(records: list[dict], plots: list[Path], base: Path):
    yield "# Training Metrics"
    yield ""
    latest = {r["split"]: r for r in records}  # the last record of each split wins
    if latest:
        yield "## Latest Metrics"
        yield ""
        for split in sorted(latest):
            record = latest[split]
            yield f"### {split}"
            yield ""
            yield f"- step: {record['step']}"
            for key in sorted(record["metrics"]):
                yield f"- {key}: {record['metrics'][key]:.6g}"
            yield ""
    if plots:
        yield "## Plots"
        yield ""
        for plot in plots:
            yield f"- [{plot.stem}]({plot.relative_to(base).as_posix()})"


def save_metrics_markdown(path, records: list[dict], plot_paths: list[Path]) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text("\n".join(_markdown(records, list(plot_paths), path.parent)).rstrip() + "\n", encoding="utf-8")
    return path


def save_metric_plots(records: list[dict], plot_dir) -> list[Path]:
    """One PNG per metric; returns the written paths (empty without matplotlib)."""
    plot_dir = Path(plot_dir)
    plot_dir.mkdir(parents=True, exist_ok=True)
    try:
        import matplotlib

        matplotlib.use("Agg")
        from matplotlib import pyplot
    except Exception as exc:  # headless box without matplotlib
        (plot_dir / "plotting_unavailable.txt").write_text(f"matplotlib unavailable: {exc}\n", encoding="utf-8")
        return []
    points = sorted((metric, r["split"], int(r["step"]), float(value))
                    for r in records for metric, value in r["metrics"].items())
    written = []
    for metric, rows in itertools.groupby(points, key=lambda p: p[0]):
        fig, ax = pyplot.subplots(figsize=(8, 4.5))
        for split, line in itertools.groupby(rows, key=lambda p: p[1]):
            line = list(line)
            ax.plot([p[2] for p in line], [p[3] for p in line], marker="o", label=split)
        ax.set(title=metric.replace("_", " ").title(), xlabel="step", ylabel=metric)
        ax.grid(True, alpha=0.3)
        ax.legend()
        fig.tight_layout()
        target = plot_dir / f"{metric}.png"
        fig.savefig(target, dpi=140)
        pyplot.close(fig)
        written.append(target)
    return written


class MetricsHistory:
    """A logger backend that keeps every record and writes the run's metric files on ``close``."""

    def __init__(self, run_dir, save_plots: bool = True):
        self.run_dir = Path(run_dir)
        self.save_plots = save_plots
        self.records: list[dict] = []
        self.config = None

    def log_config(self, config) -> None:
        self.config = config

    def log_text(self, name: str, text: str, step: int) -> None:
        pass

    def log_metrics(self, metrics: dict, step: int, split: str) -> None:
        record = make_record(metrics, step, split)
        if record is not None:
            self.records.append(record)

    def close(self) -> None:
        json_path = save_metrics_json(self.run_dir / "metrics.json", self.records, self.config)
        plots = save_metric_plots(self.records, self.run_dir / "plots") if self.save_plots else []
        save_metrics_markdown(json_path.with_suffix(".md"), self.records, plots)
