"""Tensor helpers shared by the gist strategies.

A strategy sees a chunk as ``[points, width]`` key rows (heads merged per token)
and, optionally, value rows with the same shape; it returns ``[G, width]`` key
gists and the value gists averaged over the same members.  Routing compares
gists and queries by cosine with an L2 epsilon of 1e-12.  Randomness always
comes from a private seeded CPU generator, never from the global RNG.  Results
match ``src/pra_torch/gists/common.py:14-140`` (the same reductions in the same
order, so the object path stays bit-exact against the reference).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .base import ComputedGists

NORM_EPS = 1e-12  # cosine normalisation epsilon used throughout routing
_AGGREGATIONS = ("max", "mean", "logsumexp")


@dataclass(frozen=True)
class GistScore:
    aggregate_score: float
    winning_index: int | None
    per_gist_scores: torch.Tensor | None


def _shape_error(what: str, expected: str, tensor: torch.Tensor) -> ValueError:
    return ValueError(f"{what} must be {expected}; got shape {tuple(tensor.shape)}.")


def projected_tokens(layer_tensor: torch.Tensor) -> torch.Tensor:
    """One encoded source's ``[1, heads, tokens, head_dim]`` projection as ``[tokens, heads*head_dim]``."""
    if layer_tensor.ndim != 4:
        raise _shape_error("A projected tensor", "[batch, heads, tokens, head_dim]", layer_tensor)
    if layer_tensor.shape[0] != 1:
        raise ValueError("Gists are built per independently encoded source (batch of one).")
    return layer_tensor[0].permute(1, 0, 2).reshape(layer_tensor.shape[2], -1)


def validate_points(keys: torch.Tensor, values: torch.Tensor | None) -> None:
    if keys.ndim != 2:
        raise _shape_error("Gist source keys", "[points, width]", keys)
    if values is not None and tuple(values.shape) != tuple(keys.shape):
        raise ValueError(f"Gist source values {tuple(values.shape)} must have the key shape {tuple(keys.shape)}.")


def empty_gists(keys: torch.Tensor, values: torch.Tensor | None, **metadata) -> ComputedGists:
    """No gists, with the keys' width, dtype and device."""
    k = keys.new_empty((0, int(keys.shape[-1]) if keys.ndim == 2 else 0))
    return ComputedGists(k=k, v=None if values is None else k.clone(), metadata=metadata)


def local_generator(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(int(seed))


def normalize_rows(points: torch.Tensor) -> torch.Tensor:
    """Unit rows (zero rows stay zero)."""
    return F.normalize(points, dim=-1, eps=NORM_EPS)


def assign_to_centers(points: torch.Tensor, centers: torch.Tensor, *, distance: str) -> torch.Tensor:
    """Index of each point's nearest centre (highest cosine, or smallest Euclidean distance)."""
    if distance not in ("cosine", "euclidean"):
        raise ValueError(f"Unsupported gist distance: {distance}")
    if len(centers) == 0:
        return torch.empty(len(points), dtype=torch.long, device=points.device)
    if distance == "euclidean":
        return torch.cdist(points, centers).argmin(dim=1)
    return torch.mm(normalize_rows(points), normalize_rows(centers).t()).argmax(dim=1)


def paired_means(keys, values, assignments, cluster_count):
    """Per non-empty cluster (in cluster order): the mean key, the mean value of the same
    members, the cluster id and its size."""
    clusters, members = [], []
    for cluster in range(int(cluster_count)):
        mask = assignments == cluster
        if bool(mask.any()):
            clusters.append(cluster)
            members.append(mask)
    if not clusters:
        none = empty_gists(keys, values)
        return none.k, none.v, [], []
    key_gists = torch.stack([keys[mask].mean(dim=0) for mask in members])
    value_gists = None if values is None else torch.stack([values[mask].mean(dim=0) for mask in members])
    return key_gists, value_gists, clusters, [int(mask.sum()) for mask in members]


def mean_cosine_separation(gists: torch.Tensor) -> float:
    """Average (1 - cosine) over distinct gist pairs (0 for fewer than two gists)."""
    count = int(gists.shape[0])
    if count < 2:
        return 0.0
    unit = normalize_rows(gists.detach())
    upper = torch.triu_indices(count, count, offset=1)
    return float((1.0 - (unit @ unit.t())[upper[0], upper[1]]).mean().cpu())


def reduce_scores(scores: torch.Tensor, valid: torch.Tensor | None, aggregation: str, dim: int = -1) -> torch.Tensor:
    """Masked max / mean / logsumexp along ``dim`` (invalid entries ignored)."""
    if aggregation not in _AGGREGATIONS:
        raise ValueError(f"Unsupported gist score aggregation: {aggregation}")
    valid = torch.ones_like(scores, dtype=torch.bool) if valid is None else valid
    if aggregation == "mean":
        return scores.masked_fill(~valid, 0.0).sum(dim=dim) / valid.sum(dim=dim).clamp_min(1)
    masked = scores.masked_fill(~valid, float("-inf"))
    return masked.amax(dim=dim) if aggregation == "max" else torch.logsumexp(masked, dim=dim)


def score_gist_set(query: torch.Tensor, gists: torch.Tensor, aggregation: str = "max") -> GistScore:
    """Cosine scores of one ``[width]`` query against ``[G, width]`` gists, reduced over the set."""
    if query.ndim != 1:
        raise _shape_error("A routing query", "[width]", query)
    if gists.ndim != 2:
        raise _shape_error("Routing gists", "[gists, width]", gists)
    if len(gists) == 0:
        return GistScore(float("-inf"), None, None)
    scores = normalize_rows(gists.to(query.device, query.dtype)) @ F.normalize(query, dim=-1, eps=NORM_EPS)
    winner = int(scores.argmax())
    value = scores[winner] if aggregation == "max" else reduce_scores(scores, None, aggregation, dim=0)
    return GistScore(float(value.detach().cpu()), winner, scores.detach())
