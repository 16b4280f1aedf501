"""Configuration objects for the PRA framework.

``PRAConfig`` keeps the exact field names and defaults of the reference
(``src/pra_torch/config.py:8-148``) because checkpoints serialise
``cfg.__dict__`` and must round-trip between the two frameworks.  The
validation (``__post_init__``) enforces the same accepted values
(``src/pra_torch/config.py:204-484``); the implementation is table-driven here.

``TrainConfig`` mirrors the generic loop settings of ``src/common/config.py:40-103``
plus the PRA service fields of ``src/pra_torch/config.py:529-542`` and adds the
multi-GPU knobs (``dist_*``) used by the data-parallel engine.
"""

from __future__ import annotations

import copy
import warnings
from dataclasses import dataclass, field
from pathlib import Path

import yaml

from .chunking import ChunkingConfig


# ---------------------------------------------------------------------------
# YAML helpers (same contract as src/common/config.py:12-37)
# ---------------------------------------------------------------------------

def deep_update(base: dict, updates: dict) -> dict:
    """Merge ``updates`` into ``base`` recursively (nested dicts merge, leaves replace)."""
    for key, value in updates.items():
        current = base.get(key)
        if isinstance(value, dict) and isinstance(current, dict):
            deep_update(current, value)
        else:
            base[key] = value
    return base


def read_yaml(path: str | Path) -> dict:
    """Load one YAML mapping; an empty document is an empty mapping."""
    text = Path(path).read_text(encoding="utf-8")
    payload = yaml.safe_load(text) or {}
    if not isinstance(payload, dict):
        raise TypeError(f"Expected a YAML mapping in {path}, got {type(payload).__name__}.")
    return payload


def load_yaml_config(*paths: str | Path, base: dict | None = None) -> dict:
    """Merge YAML files left to right on top of a copy of ``base``."""
    merged = copy.deepcopy(base or {})
    for path in paths:
        deep_update(merged, read_yaml(path))
    return merged


# ---------------------------------------------------------------------------
# Enumerated option tables used by PRAConfig validation
# ---------------------------------------------------------------------------

_GIST_MODES = ("mean", "last", "ref_end", "gru", "kmeans", "som", "prototype", "hybrid")
_AGGREGATIONS = ("max", "mean", "logsumexp")

_CHOICES: dict[str, tuple] = {
    "memory_transport": ("native_kv", "cross_attention"),
    "prompt_overflow_mode": ("truncate", "implicit_reference", "error"),
    "search_strategy": ("hierarchical", "reference_first", "global_chunks"),
    "routing_backend": ("tensorized", "legacy"),
    "reference_score_aggregation": _AGGREGATIONS,
    "gist_mode": _GIST_MODES,
    "gist_score_aggregation": _AGGREGATIONS,
    "reference_gist_score_aggregation": _AGGREGATIONS,
    "gist_overflow_policy": ("truncate", "merge_tail", "error"),
    "gist_kmeans_init": ("kmeans++", "sample"),
    "gist_kmeans_empty_cluster_policy": ("farthest", "error"),
    "gist_som_distance": ("cosine", "euclidean"),
    "gist_prototype_method": ("farthest",),
    "gist_prototype_init": ("mean_nearest", "sample"),
    "gist_prototype_distance": ("cosine", "euclidean"),
    "gist_hybrid_global_mode": ("mean", "last", "ref_end", "gru"),
    "gist_hybrid_local_mode": ("kmeans", "som", "prototype"),
    "chunking_mode": ("none", "fixed", "markers", "semantic"),
    "overlap_materialization": ("deduplicate", "keep_duplicates"),
    "reference_encoding_strategy": ("independent", "block_slice", "native_slice"),
    "reference_position_mode": ("local", "global"),
    "prompt_position_mode": ("local", "historical"),
    "encoding_context_mode": ("independent", "overlap", "historical_window"),
    "reference_overflow_policy": ("truncate", "error"),
    "kv_cache_residency": ("gpu", "cpu"),
    "detail_materialization": ("selected_chunks", "full_reference", "gist_only"),
    "memory_bucket_strategy": ("optimal_contiguous", "equal_count"),
    "cache_build_mode": ("detached", "trainable_gist"),
    "summary_mode": ("replace", "hybrid", "augment"),
    "recursive_cycle_policy": ("skip", "error", "link_only"),
    "recursive_missing_ref_policy": ("skip", "warn", "error"),
    "chunk_match_mode": ("exact_id", "any_overlap", "iou_threshold"),
    "model_variant": ("custom", "td_sa", "td_pra", "tdx_pra"),
}

_NON_NEGATIVE_INTS = (
    "recursive_max_depth",
    "recursive_max_total_references",
    "recursive_max_total_tokens",
    "recursive_max_children_per_reference",
)


@dataclass
class PRAConfig:
    """Architecture, routing, cache and legacy training settings.

    Field names and defaults are part of the checkpoint format (``cfg`` entry of
    ``pra_tiny.pt`` / ``latest.pt``); do not rename them.
    """

    # Decoder dimensions.
    vocab_size: int = 128
    d_model: int = 128
    n_heads: int = 4
    n_layers: int = 4
    n_vanilla_layers: int = 0
    n_mixed_layers: int = 0
    d_ff: int | None = None
    max_seq_len: int = 128
    model_max_context_tokens: int | None = None
    dropout: float = 0.0
    model_variant: str = "custom"

    # Routing budgets and transport.
    pra_layer_ids: tuple[int, ...] = (2, 3)
    top_k_references: int = 2
    top_k_chunks_per_reference: int = 1
    top_k_refs: int | None = None
    trigger_threshold: float = 0.2
    memory_transport: str = "native_kv"
    use_cross_attention_memory: bool | None = None
    use_concat_memory: bool | None = None
    memory_alpha: float = 0.5

    # Long prompts.
    max_prompt_direct_tokens: int | None = None
    prompt_overflow_mode: str = "truncate"
    max_prompt_gists: int | None = None
    max_materialized_memory_tokens: int | None = None
    context_safety_reserve_tokens: int = 0

    # Search and gists.
    search_strategy: str = "hierarchical"
    routing_backend: str = "tensorized"
    reference_score_aggregation: str = "max"
    reference_level_gist_mode: str | None = None
    reference_gists_per_reference: int = 1
    reference_gist_score_aggregation: str = "max"
    gist_mode: str = "mean"
    gists_per_chunk: int = 1
    gist_score_aggregation: str = "max"
    max_gists_per_reference: int = 4
    gist_overflow_policy: str = "truncate"
    gist_gru_hidden_size: int | None = None
    gist_gru_num_layers: int = 1
    gist_gru_bidirectional: bool = False
    ref_end_token: str = "<REF_END>"

    # Multi-gist strategies.
    gist_kmeans_max_iters: int = 8
    gist_kmeans_init: str = "kmeans++"
    gist_kmeans_tol: float = 1e-4
    gist_kmeans_normalize: bool = True
    gist_kmeans_seed: int = 0
    gist_kmeans_empty_cluster_policy: str = "farthest"
    gist_som_steps: int = 32
    gist_som_learning_rate: float = 0.2
    gist_som_final_learning_rate: float = 0.05
    gist_som_neighborhood_radius: float = 1.0
    gist_som_final_neighborhood_radius: float = 0.0
    gist_som_distance: str = "cosine"
    gist_som_normalize: bool = True
    gist_som_init: str = "sample"
    gist_som_seed: int = 0
    gist_som_topology: str = "line"
    gist_prototype_method: str = "farthest"
    gist_prototype_init: str = "mean_nearest"
    gist_prototype_refine: bool = True
    gist_prototype_normalize: bool = True
    gist_prototype_distance: str = "cosine"
    gist_prototype_seed: int = 0
    gist_hybrid_global_mode: str = "mean"
    gist_hybrid_local_mode: str = "kmeans"
    gist_hybrid_global_count: int = 1
    gist_hybrid_deduplicate: bool = True
    gist_hybrid_min_cosine_separation: float = 0.0

    # Partitioning and materialisation detail.
    chunking_mode: str = "none"
    fixed_chunk_tokens: int = 64
    fixed_chunk_overlap_tokens: int = 0
    chunk_overlap_fraction: float = 0.0
    overlap_materialization: str = "deduplicate"
    reference_encoding_strategy: str = "independent"
    encoding_block_references: int = 8
    encoding_overlap_fraction: float = 0.0
    reference_position_mode: str = "local"
    prompt_position_mode: str = "local"
    reference_overflow_policy: str = "truncate"
    kv_cache_residency: str = "gpu"
    kv_cache_pin_memory: bool = False
    kv_cache_non_blocking: bool = False
    marker_rules: tuple[str, ...] = ("<PRA_CHUNK>",)
    semantic_chunker: object | None = None
    encoding_chunking: ChunkingConfig | dict | None = None
    routing_chunking: ChunkingConfig | dict | None = None
    encoding_context_mode: str = "independent"
    detail_materialization: str = "selected_chunks"

    # Legacy cross-attention bucketing.
    memory_bucket_count: int = 1
    memory_bucket_strategy: str = "optimal_contiguous"

    # Cache construction.
    cache_build_mode: str = "detached"
    use_summary: bool = False
    summary_mode: str = "replace"

    # Recursive references.
    recursive_refs_enabled: bool = False
    recursive_max_depth: int = 2
    recursive_max_total_references: int = 16
    recursive_max_total_tokens: int = 2048
    recursive_max_children_per_reference: int = 8
    recursive_cycle_policy: str = "skip"
    recursive_missing_ref_policy: str = "warn"

    # Diagnostics.
    collect_detailed_timing: bool = False
    collect_attention_metrics: bool = True
    collect_per_head_metrics: bool = False
    collect_routing_metrics: bool = False
    collect_rank_diagnostics: bool = False
    chunk_match_mode: str = "exact_id"
    chunk_iou_threshold: float = 0.5

    # Legacy convenience fields.
    batch_size: int = 8
    lr: float = 3e-4
    steps: int = 500
    device: str = "cuda"

    # ------------------------------------------------------------------
    @property
    def effective_model_max_context_tokens(self) -> int:
        """Hard native-operation ceiling (defaults to the positional table size)."""
        return int(self.model_max_context_tokens or self.max_seq_len)

    @property
    def effective_prompt_direct_tokens(self) -> int:
        """Direct-token capacity after the safety reserve."""
        limit = self.effective_model_max_context_tokens
        wanted = self.max_prompt_direct_tokens or limit
        return min(int(wanted), int(self.max_seq_len), int(limit - self.context_safety_reserve_tokens))

    @property
    def routing_chunking_config(self) -> ChunkingConfig:
        """Routing partition policy (explicit, or migrated from the legacy fields)."""
        if self.routing_chunking is not None:
            return ChunkingConfig.from_value(self.routing_chunking)
        return ChunkingConfig(
            mode=self.chunking_mode,
            chunk_tokens=self.fixed_chunk_tokens,
            overlap_fraction=self.chunk_overlap_fraction,
            overlap_tokens=self.fixed_chunk_overlap_tokens,
            markers=tuple(self.marker_rules),
            semantic_chunker=self.semantic_chunker,
        )

    @property
    def encoding_chunking_config(self) -> ChunkingConfig:
        """Model-call partition policy; ``none`` means bounded automatically."""
        if self.encoding_chunking is not None:
            return ChunkingConfig.from_value(self.encoding_chunking)
        return ChunkingConfig(mode="none", chunk_tokens=None, overlap_fraction=self.encoding_overlap_fraction)

    @property
    def resolved_chunk_overlap_tokens(self) -> int:
        policy = self.routing_chunking_config
        return policy.resolved_overlap_tokens(policy.chunk_tokens)

    def prompt_tail_position_offset(self, head_tokens: int, direct_tokens: int) -> int:
        """Historical positions continue only while the whole history fits natively."""
        if self.prompt_position_mode != "historical":
            return 0
        if int(head_tokens) + int(direct_tokens) > self.effective_model_max_context_tokens:
            return 0
        return int(head_tokens)

    @property
    def n_pra_layers(self) -> int:
        return self.n_layers - self.n_vanilla_layers - self.n_mixed_layers

    # ------------------------------------------------------------------
    def __post_init__(self) -> None:
        self._normalise_limits()
        self._normalise_aliases()
        for name, allowed in _CHOICES.items():
            value = getattr(self, name)
            if value not in allowed:
                raise ValueError(f"Unsupported {name}: {value}")
        self._validate_gists()
        self._validate_chunking()
        self._validate_misc()
        self._apply_variant()

    def _normalise_limits(self) -> None:
        self.max_seq_len = int(self.max_seq_len)
        if self.max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive.")
        if self.model_max_context_tokens is not None:
            self.model_max_context_tokens = int(self.model_max_context_tokens)
            if self.model_max_context_tokens <= 0:
                raise ValueError("model_max_context_tokens must be positive or None.")
            if self.model_max_context_tokens > self.max_seq_len:
                raise ValueError("model_max_context_tokens cannot exceed this model's max_seq_len.")
        self.context_safety_reserve_tokens = int(self.context_safety_reserve_tokens)
        if not 0 <= self.context_safety_reserve_tokens < self.effective_model_max_context_tokens:
            raise ValueError("context_safety_reserve_tokens must fit inside the model limit.")
        for name in ("max_materialized_memory_tokens", "max_prompt_direct_tokens", "max_prompt_gists"):
            value = getattr(self, name)
            if value is not None:
                value = int(value)
                if value <= 0:
                    raise ValueError(f"{name} must be positive or None.")
                setattr(self, name, value)

    def _normalise_aliases(self) -> None:
        if self.use_cross_attention_memory is not None:
            warnings.warn("use_cross_attention_memory is deprecated; use memory_transport.",
                          DeprecationWarning, stacklevel=3)
            self.memory_transport = "cross_attention" if self.use_cross_attention_memory else "native_kv"
        if self.use_concat_memory:
            warnings.warn("use_concat_memory is deprecated; native_kv is the concatenated-K/V mode.",
                          DeprecationWarning, stacklevel=3)
            if self.memory_transport == "cross_attention":
                raise ValueError("Legacy cross-attention and concat-memory flags conflict.")
            self.memory_transport = "native_kv"
        if self.top_k_refs is not None:
            warnings.warn("top_k_refs is deprecated; use top_k_references and top_k_chunks_per_reference.",
                          DeprecationWarning, stacklevel=3)
            self.top_k_references = int(self.top_k_refs)
        self.top_k_references = int(self.top_k_references)
        self.top_k_chunks_per_reference = int(self.top_k_chunks_per_reference)
        if self.top_k_references < 0 or self.top_k_chunks_per_reference < 0:
            raise ValueError("PRA top-k values must be non-negative; zero selects nothing.")
        if self.effective_prompt_direct_tokens <= 0:
            raise ValueError("The model context reserve leaves no direct prompt capacity.")

    def _validate_gists(self) -> None:
        if self.reference_level_gist_mode not in (None, *_GIST_MODES):
            raise ValueError(f"Unsupported reference_level_gist_mode: {self.reference_level_gist_mode}")
        if self.reference_level_gist_mode == "ref_end":
            raise ValueError("reference_level_gist_mode='ref_end' has no URI-level token marker.")
        self.gists_per_chunk = int(self.gists_per_chunk)
        self.reference_gists_per_reference = int(self.reference_gists_per_reference)
        if min(self.gists_per_chunk, self.reference_gists_per_reference) <= 0:
            raise ValueError("Chunk and reference gist counts must be positive.")
        self.max_gists_per_reference = int(self.max_gists_per_reference)
        if self.max_gists_per_reference <= 0:
            raise ValueError("max_gists_per_reference must be positive.")
        self.gist_kmeans_max_iters = int(self.gist_kmeans_max_iters)
        if self.gist_kmeans_max_iters <= 0 or float(self.gist_kmeans_tol) < 0:
            raise ValueError("K-means iterations must be positive and tolerance non-negative.")
        self.gist_som_steps = int(self.gist_som_steps)
        if self.gist_som_steps < 0:
            raise ValueError("gist_som_steps must be non-negative.")
        rates = (self.gist_som_learning_rate, self.gist_som_final_learning_rate,
                 self.gist_som_neighborhood_radius, self.gist_som_final_neighborhood_radius)
        if min(float(r) for r in rates) < 0:
            raise ValueError("SOM rates and neighborhood radii must be non-negative.")
        if self.gist_som_init != "sample" or self.gist_som_topology != "line":
            raise ValueError("The current SOM implementation supports sample initialization and line topology.")
        if self.reference_level_gist_mode == "hybrid" and self.gist_hybrid_global_mode == "ref_end":
            raise ValueError("Reference-level hybrid gists cannot use a ref_end global gist.")
        self.gist_hybrid_global_count = int(self.gist_hybrid_global_count)
        if self.gist_hybrid_global_count <= 0:
            raise ValueError("gist_hybrid_global_count must be positive.")
        if not 0.0 <= float(self.gist_hybrid_min_cosine_separation) <= 2.0:
            raise ValueError("gist_hybrid_min_cosine_separation must be between zero and two.")

    def _validate_chunking(self) -> None:
        self.fixed_chunk_tokens = int(self.fixed_chunk_tokens)
        self.fixed_chunk_overlap_tokens = int(self.fixed_chunk_overlap_tokens)
        self.chunk_overlap_fraction = float(self.chunk_overlap_fraction)
        if self.fixed_chunk_tokens <= 0:
            raise ValueError("fixed_chunk_tokens must be positive.")
        if self.fixed_chunk_overlap_tokens < 0:
            raise ValueError("fixed_chunk_overlap_tokens must be non-negative.")
        if not 0.0 <= self.chunk_overlap_fraction < 1.0:
            raise ValueError("chunk_overlap_fraction must satisfy 0 <= value < 1.")
        if self.fixed_chunk_overlap_tokens and self.chunk_overlap_fraction:
            raise ValueError("Set only one of fixed_chunk_overlap_tokens and chunk_overlap_fraction.")
        if self.resolved_chunk_overlap_tokens >= self.fixed_chunk_tokens:
            raise ValueError("Resolved fixed chunk overlap must be smaller than fixed_chunk_tokens.")
        self.encoding_block_references = int(self.encoding_block_references)
        if self.encoding_block_references <= 0:
            raise ValueError("encoding_block_references must be positive.")
        self.encoding_overlap_fraction = float(self.encoding_overlap_fraction)
        if not 0.0 <= self.encoding_overlap_fraction < 1.0:
            raise ValueError("encoding_overlap_fraction must satisfy 0 <= value < 1.")
        self.encoding_chunking = (ChunkingConfig.from_value(self.encoding_chunking)
                                  if self.encoding_chunking is not None else None)
        self.routing_chunking = (ChunkingConfig.from_value(self.routing_chunking)
                                 if self.routing_chunking is not None else None)
        size = self.encoding_chunking_config.chunk_tokens
        if size is not None and size > self.effective_model_max_context_tokens:
            raise ValueError("encoding_chunking.chunk_tokens cannot exceed model_max_context_tokens.")
        self.marker_rules = tuple(str(rule) for rule in self.marker_rules)
        if self.chunking_mode == "semantic" and self.semantic_chunker is None:
            raise NotImplementedError("chunking_mode='semantic' requires an explicit semantic_chunker implementation.")

    def _validate_misc(self) -> None:
        if self.kv_cache_residency == "cpu" and self.cache_build_mode != "detached":
            raise ValueError("CPU-resident K/V requires cache_build_mode='detached'.")
        self.memory_bucket_count = int(self.memory_bucket_count)
        if self.memory_bucket_count < 0:
            raise ValueError("memory_bucket_count must be non-negative.")
        for name in _NON_NEGATIVE_INTS:
            value = int(getattr(self, name))
            if value < 0:
                raise ValueError(f"{name} must be non-negative.")
            setattr(self, name, value)
        if not 0.0 <= float(self.chunk_iou_threshold) <= 1.0:
            raise ValueError("chunk_iou_threshold must be between zero and one.")
        self.d_ff = 4 * self.d_model if self.d_ff is None else int(self.d_ff)
        if self.d_ff <= 0:
            raise ValueError("d_ff must be positive.")

    def _apply_variant(self) -> None:
        if self.model_variant == "td_sa":
            self.n_vanilla_layers, self.n_mixed_layers, self.pra_layer_ids = self.n_layers, 0, tuple()
        elif self.model_variant == "td_pra":
            self.n_vanilla_layers, self.n_mixed_layers = 0, 0
            self.pra_layer_ids = tuple(range(self.n_layers))
        elif self.model_variant == "tdx_pra":
            self.n_vanilla_layers, self.n_mixed_layers = max(self.n_layers - 2, 0), 0
            self.pra_layer_ids = tuple(range(self.n_vanilla_layers, self.n_layers))
        self.n_vanilla_layers = int(self.n_vanilla_layers)
        self.n_mixed_layers = int(self.n_mixed_layers)
        if self.n_vanilla_layers < 0 or self.n_mixed_layers < 0:
            raise ValueError("n_vanilla_layers and n_mixed_layers must be non-negative.")
        if self.n_vanilla_layers + self.n_mixed_layers > self.n_layers:
            raise ValueError("n_vanilla_layers + n_mixed_layers cannot exceed n_layers.")


# ---------------------------------------------------------------------------
# Service and training configuration
# ---------------------------------------------------------------------------

def _service_from_value(cls, value, default_type: str):
    if value is None:
        return cls()
    if isinstance(value, cls):
        return value
    if isinstance(value, str):
        return cls(type=value)
    if isinstance(value, dict):
        return cls(type=str(value.get("type", default_type)), options=dict(value.get("options") or {}))
    raise TypeError(f"Unsupported {cls.__name__} value: {value!r}")


@dataclass
class ResolverServiceConfig:
    """Which URI resolver backend to build (``in_memory`` is the only one)."""

    type: str = "in_memory"
    options: dict = field(default_factory=dict)

    @classmethod
    def from_value(cls, value) -> "ResolverServiceConfig":
        return _service_from_value(cls, value, "in_memory")


@dataclass
class CacheServiceConfig:
    """Which encoded-memory backend to build: ``simple`` (object cache) or ``paged``."""

    type: str = "simple"
    options: dict = field(default_factory=dict)

    @classmethod
    def from_value(cls, value) -> "CacheServiceConfig":
        return _service_from_value(cls, value, "simple")


@dataclass
class BaseTrainConfig:
    """Model-agnostic loop, data-loader and logging settings (``src/common/config.py:40-103``)."""

    experiment_name: str = "experiment"
    output_dir: str = "out"
    seed: int = 0
    device: str = "auto"
    dtype: str = "float32"

    epochs: int = 3
    max_steps: int | None = None
    batch_size: int = 8
    grad_accum_steps: int = 1
    learning_rate: float = 3e-4
    weight_decay: float = 0.0
    warmup_steps: int = 0
    max_grad_norm: float = 1.0

    eval_every_steps: int = 50
    save_every_steps: int = 100
    log_every_steps: int = 10
    resume_from: str | None = None
    early_stopping_patience: int | None = None

    num_workers: int = 0
    pin_memory: bool = False
    persistent_workers: bool = False
    dataset_stage: str = "dataset"
    data_dir: str = "data"
    max_examples: int | None = None
    max_seq_len: int = 96
    shuffle: bool = True

    mixed_precision: bool = False
    use_tensorboard: bool = True
    save_metric_plots: bool = True
    use_wandb: bool = False
    wandb_project: str = "transformer-experiments"
    use_clearml: bool = False
    clearml_project: str = "Transformer Experiments"

    def __post_init__(self) -> None:
        for name in ("epochs", "batch_size", "grad_accum_steps", "warmup_steps"):
            setattr(self, name, int(getattr(self, name)))
        if self.max_steps is not None:
            self.max_steps = int(self.max_steps)
        if self.epochs < 0:
            raise ValueError("epochs must be non-negative.")
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive.")
        if self.grad_accum_steps <= 0:
            raise ValueError("grad_accum_steps must be positive.")
        if self.max_steps is not None and self.max_steps < 0:
            raise ValueError("max_steps must be non-negative when configured.")
        if self.warmup_steps < 0:
            raise ValueError("warmup_steps must be non-negative.")


@dataclass
class TrainConfig(BaseTrainConfig):
    """Training settings with PRA resolver/cache services."""

    experiment_name: str = "standalone_tiny"
    dataset_stage: str = "stage0_synthetic_memory"
    resolver_config: ResolverServiceConfig = field(default_factory=ResolverServiceConfig)
    cache_config: CacheServiceConfig = field(default_factory=CacheServiceConfig)

    def __post_init__(self) -> None:
        super().__post_init__()
        self.resolver_config = ResolverServiceConfig.from_value(self.resolver_config)
        self.cache_config = CacheServiceConfig.from_value(self.cache_config)


__all__ = [
    "BaseTrainConfig",
    "CacheServiceConfig",
    "PRAConfig",
    "ResolverServiceConfig",
    "TrainConfig",
    "deep_update",
    "load_yaml_config",
    "read_yaml",
]
