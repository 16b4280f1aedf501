"""Derived metrics for fixed-target native-KV experiments (``src/pra_torch/native_metrics.py``)."""

from __future__ import annotations

import math
from collections.abc import Mapping

RCB_EPSILON = 1e-8
_REQUIRED = ("sa_full", "sa_tail", "native_all", "native_oracle", "native_routed", "native_shuffled",
             "native_disabled")


def recovered_context_benefit(*, sa_full_loss: float, sa_tail_loss: float, pra_loss: float,
                              epsilon: float = RCB_EPSILON) -> float | None:
    """Fraction of the dense-context benefit PRA recovers (unclamped; ``None`` when undefined)."""
    gain = float(sa_tail_loss) - float(sa_full_loss)
    if abs(gain) <= epsilon:
        return None
    return (float(sa_tail_loss) - float(pra_loss)) / gain


def derive_native_kv_metrics(losses: Mapping[str, float]) -> dict[str, float | None]:
    missing = sorted(set(_REQUIRED) - set(losses))
    if missing:
        raise ValueError(f"Missing native-KV conditions: {', '.join(missing)}")
    v = {k: float(x) for k, x in losses.items()}
    out: dict[str, float | None] = {
        "transport_gap": v["native_all"] - v["sa_full"], "sparse_gap": v["native_oracle"] - v["native_all"],
        "routing_gap": v["native_routed"] - v["native_oracle"], "full_context_benefit": v["sa_tail"] - v["sa_full"],
        "dependency_gain": v["sa_tail"] - v["sa_full"],
        "content_causality_oracle": v["native_shuffled"] - v["native_oracle"],
        "content_causality_routed": v["native_shuffled"] - v["native_routed"],
        "disabled_wrapper_gap": v["native_disabled"] - v["sa_tail"],
    }
    for cond in ("all", "oracle", "routed", "shuffled"):
        out[f"memory_benefit_{cond}"] = v["sa_tail"] - v[f"native_{cond}"]
        out[f"rcb_{cond}"] = recovered_context_benefit(sa_full_loss=v["sa_full"], sa_tail_loss=v["sa_tail"],
                                                       pra_loss=v[f"native_{cond}"])
    return out


def finite_values(values):
    return [float(x) for x in values if x is not None and math.isfinite(float(x))]
