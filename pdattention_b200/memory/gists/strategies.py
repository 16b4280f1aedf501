"""Single- and multi-gist strategies (per-chunk definitions; CPU path and oracle)."""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.nn.utils.rnn import pack_padded_sequence

from .base import ComputedGists, GistContext
from .common import (
    assign_to_centers,
    empty_gists,
    local_generator,
    mean_cosine_separation,
    normalize_rows,
    paired_means,
    validate_points,
)


class GRUGistPooler(nn.Module):
    """Learned recurrent reduction ``[B,T,D] -> [B,D]`` (parameter names match the checkpoint layout)."""

    def __init__(self, d_model: int, hidden_size: int | None = None, num_layers: int = 1,
                 bidirectional: bool = False, dropout: float = 0.0):
        super().__init__()
        hidden = int(hidden_size or d_model)
        self.bidirectional = bool(bidirectional)
        self.gru = nn.GRU(input_size=d_model, hidden_size=hidden, num_layers=int(num_layers), batch_first=True,
                          bidirectional=self.bidirectional, dropout=float(dropout) if int(num_layers) > 1 else 0.0)
        self.output = nn.Linear(hidden * (2 if self.bidirectional else 1), d_model)

    def forward(self, token_keys: torch.Tensor, lengths: torch.Tensor | None = None) -> torch.Tensor:
        if token_keys.ndim != 3:
            raise ValueError(f"Expected token keys [batch,tokens,model], got {token_keys.shape}.")
        source = token_keys
        if lengths is not None:
            source = pack_padded_sequence(token_keys, lengths.detach().cpu(), batch_first=True, enforce_sorted=False)
        _, hidden = self.gru(source)
        pooled = torch.cat((hidden[-2], hidden[-1]), dim=-1) if self.bidirectional else hidden[-1]
        return self.output(pooled)


class SingleGistStrategy:
    """``mean`` / ``last`` / ``ref_end`` / ``gru``: exactly one gist."""

    def __init__(self, mode: str):
        self.mode = mode

    @staticmethod
    def _marker_position(context: GistContext) -> int:
        if context.tokenizer is None:
            raise ValueError("ref_end gist mode requires a tokenizer.")
        marker = context.tokenizer.encode(context.ref_end_token)
        if len(marker) != 1:
            raise ValueError(f"Reference terminator {context.ref_end_token!r} is not one atomic token.")
        hits = [i for i, t in enumerate(context.token_ids) if t == marker[0]]
        if len(hits) != 1:
            raise ValueError(f"Expected exactly one {context.ref_end_token!r} token, found {len(hits)}.")
        return hits[0]

    def pool(self, points: torch.Tensor, context: GistContext) -> torch.Tensor:
        if self.mode == "mean":
            return points.mean(dim=0)
        if self.mode == "last":
            return points[-1]
        if self.mode == "ref_end":
            return points[self._marker_position(context)]
        if self.mode == "gru":
            if context.gru_pooler is None:
                raise ValueError("gist_mode='gru' requires the model's registered GRU pooler.")
            lengths = torch.tensor([points.shape[0]], device=points.device)
            return context.gru_pooler(points.unsqueeze(0), lengths=lengths).squeeze(0)
        raise ValueError(f"Unsupported single-gist mode: {self.mode}")

    def compute(self, *, keys, values, num_gists, config, context) -> ComputedGists:
        validate_points(keys, values)
        if keys.shape[0] == 0:
            return empty_gists(keys, values, mode=self.mode, requested_gists=int(num_gists), actual_gists=0)
        k = self.pool(keys, context).unsqueeze(0)
        v = self.pool(values, context).unsqueeze(0) if values is not None else None
        return ComputedGists(k=k, v=v, metadata={
            "mode": self.mode, "requested_gists": int(num_gists), "actual_gists": 1,
            "occupancy": [int(keys.shape[0])], "mean_cosine_separation": mean_cosine_separation(k)})


def kmeanspp_random_stream(points: int, count: int, seed: int, dtype=torch.float32):
    """The random draws a seeded kmeans++ init consumes, in order.

    kmeans++ draws the first centre with ``randint(points)`` and each further
    centre with one ``multinomial(probabilities, 1)`` from a private CPU
    generator.  Without replacement, a single multinomial draw equals
    ``argmax(p / e)`` with ``e ~ Exp(1)`` of the same length and dtype drawn from
    the same generator; so the whole stream is data independent and can be
    precomputed once and shipped to a batched device kernel.

    Returns ``(first_index, exp_draws)`` with ``exp_draws`` of shape
    ``[count - 1, points]``.
    """
    gen = local_generator(seed)
    first = int(torch.randint(points, (1,), generator=gen).item())
    draws = [torch.empty(points, dtype=dtype).exponential_(1, generator=gen) for _ in range(max(count - 1, 0))]
    exp = torch.stack(draws) if draws else torch.empty((0, points), dtype=dtype)
    return first, exp


class KMeansGistStrategy:
    """Lloyd in key space; values are averaged over the same assignments."""

    @staticmethod
    def initial_centers(points: torch.Tensor, count: int, config) -> torch.Tensor:
        gen = local_generator(config.gist_kmeans_seed)
        n = points.shape[0]
        if config.gist_kmeans_init == "sample":
            order = torch.randperm(n, generator=gen)[:count]
            return points[order.to(points.device)].clone()
        if config.gist_kmeans_init != "kmeans++":
            raise ValueError(f"Unsupported k-means initialization: {config.gist_kmeans_init}")
        chosen = [int(torch.randint(n, (1,), generator=gen).item())]
        while len(chosen) < count:
            picked = torch.tensor(chosen, device=points.device)
            dist2 = torch.cdist(points, points[picked]).pow(2).min(dim=1).values
            dist2[picked] = 0
            total = float(dist2.sum().detach().cpu())
            unused = next(i for i in range(n) if i not in chosen)
            if total <= 0:
                chosen.append(unused)
                continue
            nxt = int(torch.multinomial(dist2.detach().cpu() / total, 1, generator=gen).item())
            chosen.append(unused if nxt in chosen else nxt)
        return points[torch.tensor(chosen, device=points.device)].clone()

    def compute(self, *, keys, values, num_gists, config, context) -> ComputedGists:
        del context
        validate_points(keys, values)
        requested = int(num_gists)
        count = min(max(requested, 0), int(keys.shape[0]))
        if count == 0:
            return empty_gists(keys, values, mode="kmeans", requested_gists=requested, actual_gists=0)
        work = normalize_rows(keys) if config.gist_kmeans_normalize else keys
        centers = self.initial_centers(work, count, config)
        iterations = 0
        for iterations in range(1, int(config.gist_kmeans_max_iters) + 1):
            assign = assign_to_centers(work, centers, distance="euclidean")
            rows = []
            for c in range(count):
                members = work[assign == c]
                if members.shape[0]:
                    rows.append(members.mean(dim=0))
                elif config.gist_kmeans_empty_cluster_policy == "error":
                    raise ValueError(f"Empty k-means cluster {c}.")
                else:
                    rows.append(work[int(torch.cdist(work, centers).min(dim=1).values.argmax().item())])
            updated = torch.stack(rows)
            shift = float((updated - centers).norm(dim=1).max().detach().cpu())
            centers = updated
            if shift <= float(config.gist_kmeans_tol):
                break
        assign = assign_to_centers(work, centers, distance="euclidean")
        gist_k, gist_v, _, occupancy = paired_means(keys, values, assign, count)
        if config.gist_kmeans_normalize and gist_k.shape[0]:
            gist_k = normalize_rows(gist_k)
        return ComputedGists(k=gist_k, v=gist_v, metadata={
            "mode": "kmeans", "requested_gists": requested, "actual_gists": int(gist_k.shape[0]),
            "occupancy": occupancy, "iterations": iterations, "mean_cosine_separation": mean_cosine_separation(gist_k)})


class SOMGistStrategy:
    """Line-topology self-organising map; values paired through winner assignments."""

    def compute(self, *, keys, values, num_gists, config, context) -> ComputedGists:
        del context
        validate_points(keys, values)
        requested = int(num_gists)
        count = min(max(requested, 0), int(keys.shape[0]))
        if count == 0:
            return empty_gists(keys, values, mode="som", requested_gists=requested, actual_gists=0)
        if config.gist_som_topology != "line":
            raise ValueError(f"Unsupported SOM topology: {config.gist_som_topology}")
        if config.gist_som_init != "sample":
            raise ValueError(f"Unsupported SOM initialization: {config.gist_som_init}")
        work = normalize_rows(keys) if config.gist_som_normalize else keys
        gen = local_generator(config.gist_som_seed)
        protos = work[torch.randperm(work.shape[0], generator=gen)[:count].to(work.device)].clone()
        steps = int(config.gist_som_steps)
        grid = torch.arange(count, device=work.device, dtype=work.dtype)
        for step in range(steps):
            point = work[int(torch.randint(work.shape[0], (1,), generator=gen).item())]
            win = int(assign_to_centers(point.unsqueeze(0), protos, distance=config.gist_som_distance)[0].item())
            t = step / max(steps - 1, 1)
            rate = float(config.gist_som_learning_rate) * (1 - t) + float(config.gist_som_final_learning_rate) * t
            radius = (float(config.gist_som_neighborhood_radius) * (1 - t)
                      + float(config.gist_som_final_neighborhood_radius) * t)
            if radius > 0:
                pull = torch.exp(-((grid - win) ** 2) / (2.0 * radius ** 2))
            else:
                pull = (grid == win).to(work.dtype)
            protos = protos + rate * pull[:, None] * (point - protos)
            if config.gist_som_normalize:
                protos = normalize_rows(protos)
        assign = assign_to_centers(work, protos, distance=config.gist_som_distance)
        _, gist_v, occupied, occupancy = paired_means(keys, values, assign, count)
        gist_k = protos[torch.tensor(occupied, device=protos.device, dtype=torch.long)]
        if config.gist_som_normalize and gist_k.shape[0]:
            gist_k = normalize_rows(gist_k)
        return ComputedGists(k=gist_k, v=gist_v, metadata={
            "mode": "som", "requested_gists": requested, "actual_gists": int(gist_k.shape[0]),
            "occupancy": occupancy, "steps": steps, "mean_cosine_separation": mean_cosine_separation(gist_k)})


class PrototypeGistStrategy:
    """Farthest-point representatives in (normalised) key space."""

    def compute(self, *, keys, values, num_gists, config, context) -> ComputedGists:
        del context
        validate_points(keys, values)
        requested = int(num_gists)
        count = min(max(requested, 0), int(keys.shape[0]))
        if count == 0:
            return empty_gists(keys, values, mode="prototype", requested_gists=requested, actual_gists=0)
        if config.gist_prototype_method != "farthest":
            raise ValueError(f"Unsupported prototype method: {config.gist_prototype_method}")
        work = normalize_rows(keys) if config.gist_prototype_normalize else keys
        if config.gist_prototype_init == "mean_nearest":
            first = int(torch.cdist(work, work.mean(dim=0, keepdim=True)).argmin().item())
        elif config.gist_prototype_init == "sample":
            first = int(torch.randint(work.shape[0], (1,), generator=local_generator(config.gist_prototype_seed)).item())
        else:
            raise ValueError(f"Unsupported prototype initialization: {config.gist_prototype_init}")
        picked = [first]
        while len(picked) < count:
            index = torch.tensor(picked, device=work.device)
            far = torch.cdist(work, work[index]).min(dim=1).values
            far[index] = -1
            picked.append(int(far.argmax().item()))
        assign = assign_to_centers(work, work[torch.tensor(picked, device=work.device)],
                                   distance=config.gist_prototype_distance)
        mean_k, gist_v, occupied, occupancy = paired_means(keys, values, assign, count)
        if config.gist_prototype_refine:
            gist_k = mean_k
        else:
            gist_k = keys[torch.tensor(picked, device=keys.device)][occupied]
        if config.gist_prototype_normalize and gist_k.shape[0]:
            gist_k = normalize_rows(gist_k)
        return ComputedGists(k=gist_k, v=gist_v, metadata={
            "mode": "prototype", "requested_gists": requested, "actual_gists": int(gist_k.shape[0]),
            "occupancy": occupancy, "selected_point_indices": [picked[i] for i in occupied],
            "mean_cosine_separation": mean_cosine_separation(gist_k)})


class HybridGistStrategy:
    """A global single gist followed by local multi-gist prototypes, de-duplicated."""

    _LOCAL = {"kmeans": KMeansGistStrategy, "som": SOMGistStrategy, "prototype": PrototypeGistStrategy}

    @staticmethod
    def _deduplicate(k, v, minimum_separation: float):
        if k.shape[0] < 2:
            return k, v
        kept = [0]
        for i in range(1, k.shape[0]):
            sims = F.normalize(k[i:i + 1], dim=-1) @ F.normalize(k[torch.tensor(kept, device=k.device)], dim=-1).T
            if bool(((1.0 - sims) > minimum_separation + 1e-7).all()):
                kept.append(i)
        index = torch.tensor(kept, device=k.device)
        return k[index], (v[index] if v is not None else None)

    def compute(self, *, keys, values, num_gists, config, context) -> ComputedGists:
        validate_points(keys, values)
        requested = int(num_gists)
        if requested <= 0 or keys.shape[0] == 0:
            return empty_gists(keys, values, mode="hybrid", requested_gists=requested, actual_gists=0)
        target = min(requested, int(keys.shape[0]))
        head = SingleGistStrategy(config.gist_hybrid_global_mode).compute(
            keys=keys, values=values, num_gists=min(int(config.gist_hybrid_global_count), target), config=config,
            context=context)
        local_cls = self._LOCAL.get(config.gist_hybrid_local_mode)
        if local_cls is None:
            raise ValueError(f"Unsupported hybrid local mode: {config.gist_hybrid_local_mode}")
        tail = local_cls().compute(keys=keys, values=values, num_gists=max(target - int(head.k.shape[0]), 0),
                                   config=config, context=context)
        gist_k = torch.cat((head.k, tail.k), dim=0)
        if head.v is not None and tail.v is not None:
            gist_v = torch.cat((head.v, tail.v), dim=0)
        else:
            gist_v = head.v if tail.k.shape[0] == 0 else None
        if config.gist_hybrid_deduplicate:
            gist_k, gist_v = self._deduplicate(gist_k, gist_v, float(config.gist_hybrid_min_cosine_separation))
        return ComputedGists(k=gist_k, v=gist_v, metadata={
            "mode": "hybrid", "requested_gists": requested, "actual_gists": int(gist_k.shape[0]),
            "global_mode": config.gist_hybrid_global_mode, "local_mode": config.gist_hybrid_local_mode,
            "global_metadata": head.metadata, "local_metadata": tail.metadata,
            "mean_cosine_separation": mean_cosine_separation(gist_k)})


_SINGLE = {"mean", "last", "ref_end", "gru"}
_MULTI = {"kmeans": KMeansGistStrategy, "som": SOMGistStrategy, "prototype": PrototypeGistStrategy,
          "hybrid": HybridGistStrategy}


def compute_gists(*, keys, values, mode, num_gists, config, context) -> ComputedGists:
    """Dispatch one gist construction to its strategy."""
    if mode in _SINGLE:
        strategy = SingleGistStrategy(mode)
    elif mode in _MULTI:
        strategy = _MULTI[mode]()
    else:
        raise ValueError(f"Unsupported gist mode: {mode}")
    return strategy.compute(keys=keys, values=values, num_gists=num_gists, config=config, context=context)
