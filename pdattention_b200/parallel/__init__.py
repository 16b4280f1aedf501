"""Parallelism: process groups, peer-memory collectives, data / tensor parallel engines."""

from .dist import barrier, destroy, max_over_ranks, maybe_init_distributed, world_info

__all__ = ["barrier", "destroy", "max_over_ranks", "maybe_init_distributed", "world_info"]
