"""Routing-gist strategies: compress a chunk's ``[N,D]`` projected keys (and the
paired values under the same assignments) into ``[G,D]`` gists.

Strategy semantics follow ``src/pra_torch/gists/`` of the reference:

* ``mean`` / ``last`` / ``ref_end`` / ``gru`` -- one gist (``single.py:59-119``);
* ``kmeans`` -- Lloyd in (optionally L2-normalised) key space, kmeans++ or
  sampled init from a local seeded CPU generator, farthest-point reseed of
  empty clusters, value gists paired through the same assignments
  (``kmeans.py:19-95``);
* ``som`` -- a line-topology self-organising map (``som.py:19-85``);
* ``prototype`` -- farthest-point representatives (``prototype.py:19-67``);
* ``hybrid`` -- a global single gist followed by local prototypes, with
  near-duplicate removal (``hybrid.py:16-91``).

The batched GPU path for the hot modes (mean, kmeans) lives in
``pdattention_b200.ops.gist``; these per-chunk implementations are the
readable definitions and the CPU path.
"""

from .base import ComputedGists, GistContext, GistStrategy
from .common import GistScore, projected_tokens, score_gist_set
from .strategies import (
    GRUGistPooler,
    HybridGistStrategy,
    KMeansGistStrategy,
    PrototypeGistStrategy,
    SingleGistStrategy,
    SOMGistStrategy,
    compute_gists,
    kmeanspp_random_stream,
)

__all__ = [
    "ComputedGists",
    "GRUGistPooler",
    "GistContext",
    "GistScore",
    "GistStrategy",
    "HybridGistStrategy",
    "KMeansGistStrategy",
    "PrototypeGistStrategy",
    "SOMGistStrategy",
    "SingleGistStrategy",
    "compute_gists",
    "kmeanspp_random_stream",
    "projected_tokens",
    "score_gist_set",
]
