"""Gist strategy contract: ``[N,D]`` points -> ``ComputedGists`` with ``k``/``v`` of shape ``[G,D]``."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Protocol, Sequence

import torch


@dataclass(frozen=True)
class GistContext:
    level: str
    token_ids: Sequence[int] = ()
    tokenizer: Any = None
    ref_end_token: str = "<REF_END>"
    gru_pooler: Any = None


@dataclass
class ComputedGists:
    k: torch.Tensor
    v: torch.Tensor | None = None
    metadata: dict[str, Any] = field(default_factory=dict)


class GistStrategy(Protocol):
    def compute(self, *, keys: torch.Tensor, values: torch.Tensor | None, num_gists: int, config: Any,
                context: GistContext) -> ComputedGists:
        ...
