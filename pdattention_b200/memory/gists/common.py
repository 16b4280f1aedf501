"""Shared gist helpers: head merging, normalisation, assignment, paired means, scoring."""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .base import ComputedGists

NORM_EPS = 1e-12  # cosine normalisation epsilon used throughout routing


@dataclass(frozen=True)
class GistScore:
    aggregate_score: float
    winning_index: int | None
    per_gist_scores: torch.Tensor | None


def projected_tokens(layer_tensor: torch.Tensor) -> torch.Tensor:
    """``[1,H,T,Dh]`` per-head projections -> ``[T,H*Dh]`` token rows."""
    if layer_tensor.ndim != 4:
        raise ValueError(f"Expected projected tensor [batch,heads,tokens,head_dim], got {tuple(layer_tensor.shape)}.")
    if layer_tensor.shape[0] != 1:
        raise ValueError("Gist construction expects one independently encoded source.")
    return layer_tensor[0].transpose(0, 1).reshape(layer_tensor.shape[2], -1)


def validate_points(keys: torch.Tensor, values: torch.Tensor | None) -> None:
    if keys.ndim != 2:
        raise ValueError(f"Expected gist source keys [points,model], got {tuple(keys.shape)}.")
    if values is not None and (values.ndim != 2 or values.shape != keys.shape):
        raise ValueError(f"Gist source values must match key shape exactly: {tuple(values.shape)} != {tuple(keys.shape)}.")


def empty_gists(keys: torch.Tensor, values: torch.Tensor | None, **metadata) -> ComputedGists:
    width = int(keys.shape[-1]) if keys.ndim == 2 else 0
    empty = keys.new_empty((0, width))
    return ComputedGists(k=empty, v=empty.clone() if values is not None else None, metadata=metadata)


def local_generator(seed: int) -> torch.Generator:
    """A private CPU generator: strategies never consume global RNG state."""
    return torch.Generator(device="cpu").manual_seed(int(seed))


def normalize_rows(points: torch.Tensor) -> torch.Tensor:
    return F.normalize(points, dim=-1, eps=NORM_EPS)


def assign_to_centers(points: torch.Tensor, centers: torch.Tensor, *, distance: str) -> torch.Tensor:
    if centers.shape[0] == 0:
        return torch.empty(points.shape[0], dtype=torch.long, device=points.device)
    if distance == "cosine":
        return (normalize_rows(points) @ normalize_rows(centers).T).argmax(dim=1)
    if distance == "euclidean":
        return torch.cdist(points, centers).argmin(dim=1)
    raise ValueError(f"Unsupported gist distance: {distance}")


def paired_means(keys, values, assignments, cluster_count):
    """Per occupied cluster: mean key, mean value (same members), cluster ids, sizes."""
    occupied = [c for c in range(int(cluster_count)) if bool((assignments == c).any())]
    if not occupied:
        empty = empty_gists(keys, values)
        return empty.k, empty.v, [], []
    members = [assignments == c for c in occupied]
    key_gists = torch.stack([keys[m].mean(dim=0) for m in members])
    value_gists = torch.stack([values[m].mean(dim=0) for m in members]) if values is not None else None
    return key_gists, value_gists, occupied, [int(m.sum().item()) for m in members]


def mean_cosine_separation(gists: torch.Tensor) -> float:
    if gists.shape[0] < 2:
        return 0.0
    unit = normalize_rows(gists.detach())
    sim = unit @ unit.T
    i, j = torch.triu_indices(gists.shape[0], gists.shape[0], offset=1)
    return float((1.0 - sim[i, j]).mean().cpu())


def reduce_scores(scores: torch.Tensor, valid: torch.Tensor | None, aggregation: str, dim: int = -1) -> torch.Tensor:
    """Masked max / mean / logsumexp along ``dim`` (invalid entries ignored)."""
    if valid is None:
        valid = torch.ones_like(scores, dtype=torch.bool)
    if aggregation == "max":
        return scores.masked_fill(~valid, float("-inf")).amax(dim=dim)
    if aggregation == "mean":
        return scores.masked_fill(~valid, 0.0).sum(dim=dim) / valid.sum(dim=dim).clamp_min(1)
    if aggregation == "logsumexp":
        return torch.logsumexp(scores.masked_fill(~valid, float("-inf")), dim=dim)
    raise ValueError(f"Unsupported gist score aggregation: {aggregation}")


def score_gist_set(query: torch.Tensor, gists: torch.Tensor, aggregation: str = "max") -> GistScore:
    """Cosine-score one ``[D]`` query against ``[G,D]`` gists and reduce the set."""
    if query.ndim != 1:
        raise ValueError(f"Expected one routing query [model], got {tuple(query.shape)}.")
    if gists.ndim != 2:
        raise ValueError(f"Expected routing gists [gists,model], got {tuple(gists.shape)}.")
    if gists.shape[0] == 0:
        return GistScore(float("-inf"), None, None)
    scores = normalize_rows(gists.to(query.device, query.dtype)) @ F.normalize(query, dim=-1, eps=NORM_EPS)
    winner = int(scores.argmax().item())
    if aggregation == "max":
        value = scores[winner]
    else:
        value = reduce_scores(scores, None, aggregation, dim=0)
    return GistScore(float(value.detach().cpu()), winner, scores.detach())
