"""Metric history persistence: ``metrics.json``, ``metrics.md`` and headless PNG plots
(``src/common/plots.py``; ``plotting_unavailable.txt`` when matplotlib is absent)."""

from __future__ import annotations

import json
from collections import defaultdict
from dataclasses import asdict, is_dataclass
from pathlib import Path

_RECORD_DIMENSIONS = {"epoch", "batch_in_epoch", "batch_step", "optimizer_step", "optimizer_updated", "batches"}


def _plain(config):
    if is_dataclass(config):
        return asdict(config)
    if hasattr(config, "__dict__"):
        return dict(config.__dict__)
    return dict(config) if isinstance(config, dict) else str(config)


def save_metrics_json(path, records: list[dict], config=None) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps({"config": _plain(config), "records": records}, indent=2, default=str), encoding="utf-8")
    return path


def save_metrics_markdown(path, records: list[dict], plot_paths: list[Path]) -> Path:
    path = Path(path)
    latest = {}
    for record in records:
        latest[record["split"]] = record
    lines = ["# Training Metrics", ""]
    if latest:
        lines += ["## Latest Metrics", ""]
        for split, record in sorted(latest.items()):
            lines += [f"### {split}", "", f"- step: {record['step']}"]
            lines += [f"- {k}: {v:.6g}" for k, v in sorted(record["metrics"].items())]
            lines.append("")
    if plot_paths:
        lines += ["## Plots", ""]
        lines += [f"- [{p.stem}]({p.relative_to(path.parent).as_posix()})" for p in plot_paths]
    path.write_text("\n".join(lines).rstrip() + "\n", encoding="utf-8")
    return path


def save_metric_plots(records: list[dict], plot_dir) -> list[Path]:
    plot_dir = Path(plot_dir)
    plot_dir.mkdir(parents=True, exist_ok=True)
    series = defaultdict(lambda: defaultdict(list))
    for record in records:
        for key, value in record["metrics"].items():
            series[key][record["split"]].append((int(record["step"]), float(value)))
    try:
        import matplotlib

        matplotlib.use("Agg")
        import matplotlib.pyplot as plt
    except Exception as exc:
        (plot_dir / "plotting_unavailable.txt").write_text(f"matplotlib unavailable: {exc}\n", encoding="utf-8")
        return []
    out = []
    for metric, splits in sorted(series.items()):
        fig, ax = plt.subplots(figsize=(8, 4.5))
        for split, values in sorted(splits.items()):
            values = sorted(values)
            ax.plot([s for s, _ in values], [v for _, v in values], marker="o", label=split)
        ax.set_title(metric.replace("_", " ").title())
        ax.set_xlabel("step")
        ax.set_ylabel(metric)
        ax.grid(True, alpha=0.3)
        ax.legend()
        fig.tight_layout()
        target = plot_dir / f"{metric}.png"
        fig.savefig(target, dpi=140)
        plt.close(fig)
        out.append(target)
    return out


class MetricsHistory:
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
        scalars = {k: float(v) for k, v in metrics.items() if isinstance(v, (int, float))}
        dims = {k: scalars.pop(k) for k in list(scalars) if k in _RECORD_DIMENSIONS}
        if scalars:
            self.records.append({"step": int(step), "split": str(split), **dims, "metrics": scalars})

    def close(self) -> None:
        target = save_metrics_json(self.run_dir / "metrics.json", self.records, self.config)
        plots = save_metric_plots(self.records, self.run_dir / "plots") if self.save_plots else []
        save_metrics_markdown(target.with_suffix(".md"), self.records, plots)
