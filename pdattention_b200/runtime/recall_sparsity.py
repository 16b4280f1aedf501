"""Recall as a function of the selected candidate fraction (``src/common/recall_sparsity.py``).

For each fraction ``f`` every example selects its top ``ceil(f * N_i)``
candidates; recall / any / all evidence recall and the exact selected K/V
token fraction (when token lengths are given) are averaged.  Also reported:
the smallest fraction reaching 70/80/90/95% recall, the normalised area under
the curve up to 30%, and fixed-``k`` cut-offs.
"""

from __future__ import annotations

import math
import statistics
from collections.abc import Hashable, Sequence

DEFAULT_FRACTIONS = (0.01, 0.02, 0.05, 0.10, 0.15, 0.20, 0.25, 0.30, 0.50, 1.0)
DEFAULT_FIXED_K = (1, 3, 8, 16)


def _check(rankings, evidence, sizes, lengths) -> None:
    if not rankings or len(rankings) != len(evidence):
        raise ValueError("Rankings and evidence_ids must contain the same non-zero example count.")
    if sizes is not None and len(sizes) != len(rankings):
        raise ValueError("candidate_sizes must contain one value per ranking.")
    if lengths is not None and len(lengths) != len(rankings):
        raise ValueError("candidate_token_lengths must contain one row per ranking.")
    for i, (ranking, ev) in enumerate(zip(rankings, evidence)):
        if not ranking or not ev:
            raise ValueError(f"Example {i} must have candidates and evidence.")
        if len(set(ranking)) != len(ranking):
            raise ValueError(f"Example {i} ranking contains duplicate identities.")
        if sizes is not None and int(sizes[i]) != len(ranking):
            raise ValueError(f"Example {i} candidate size does not match its ranking.")
        if lengths is not None and (len(lengths[i]) != len(ranking) or any(int(x) <= 0 for x in lengths[i])):
            raise ValueError(f"Example {i} requires one positive token length per candidate.")


def _at_cutoffs(rankings, evidence, cutoffs, lengths) -> dict:
    rec, any_r, all_r, frac, kv = [], [], [], [], []
    for i, (ranking, ev, cut) in enumerate(zip(rankings, evidence, cutoffs)):
        hits = len(set(ranking[: int(cut)]) & ev)
        rec.append(hits / len(ev))
        any_r.append(float(hits > 0))
        all_r.append(float(hits == len(ev)))
        frac.append(min(int(cut), len(ranking)) / len(ranking))
        if lengths is not None:
            kv.append(sum(lengths[i][: int(cut)]) / sum(lengths[i]))
    return {"recall": statistics.fmean(rec), "any_evidence_recall": statistics.fmean(any_r),
            "all_evidence_recall": statistics.fmean(all_r), "selected_chunk_fraction": statistics.fmean(frac),
            "selected_kv_token_fraction": statistics.fmean(kv) if kv else None}


def _sparse_auc(curve, limit: float = 0.30) -> float:
    pts = [(0.0, 0.0)] + [(float(r["fraction"]), float(r["recall"])) for r in curve if float(r["fraction"]) <= limit]
    if pts[-1][0] != limit:
        raise ValueError(f"Recall curve must include fraction {limit:.2f} for sparse AUC.")
    return sum((x1 - x0) * (y0 + y1) / 2 for (x0, y0), (x1, y1) in zip(pts, pts[1:])) / limit


def recall_sparsity_curve(rankings: Sequence[Sequence[Hashable]], evidence_ids: Sequence[set[Hashable]], *,
                          candidate_sizes=None, fractions=DEFAULT_FRACTIONS, fixed_k=DEFAULT_FIXED_K,
                          candidate_token_lengths=None, require_complete_endpoint: bool = False) -> dict:
    _check(rankings, evidence_ids, candidate_sizes, candidate_token_lengths)
    fracs = sorted({float(f) for f in fractions})
    if not fracs or any(f <= 0.0 or f > 1.0 for f in fracs):
        raise ValueError("Fractions must lie in (0, 1].")
    curve = [{"fraction": f, **_at_cutoffs(rankings, evidence_ids,
                                           [max(1, math.ceil(f * len(r))) for r in rankings],
                                           candidate_token_lengths)} for f in fracs]
    recalls = [float(r["recall"]) for r in curve]
    if any(a > b + 1e-12 for a, b in zip(recalls, recalls[1:])):
        raise AssertionError("Recall-sparsity curve is not monotonic.")
    complete = bool(curve[-1]["fraction"] == 1.0 and abs(recalls[-1] - 1.0) <= 1e-12)
    if require_complete_endpoint and not complete:
        raise AssertionError("Selecting 100% of indexed candidates does not recover all evidence.")
    inverse = {f"f{int(t * 100)}": next((float(r["selected_chunk_fraction"]) for r in curve if float(r["recall"]) >= t),
                                        None) for t in (0.70, 0.80, 0.90, 0.95)}
    fixed = {}
    for k in sorted({int(v) for v in fixed_k}):
        if k <= 0:
            raise ValueError("Fixed-k values must be positive.")
        fixed[str(k)] = _at_cutoffs(rankings, evidence_ids, [min(k, len(r)) for r in rankings], candidate_token_lengths)
    return {"examples": len(rankings), "curve": curve, "inverse": inverse, "auc_0_30": _sparse_auc(curve),
            "fixed_k": fixed, "endpoint_complete": complete,
            "evidence_semantics": "fraction of mapped evidence identities recovered",
            "kv_fraction_exact": candidate_token_lengths is not None}
