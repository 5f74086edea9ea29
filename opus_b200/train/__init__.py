"""Scoring and selection (drop-in for OPUS.train, OPUS/train/__init__.py:8-27)."""
from .data_selection import (
    compute_GradProd_GC_per_iter,
    find_GClayers,
    get_batch_opus,
    greedy_selection,
    initialize_projector,
    stochastic_greedy_selection,
)
from .random_projection import GradientProjector

__all__ = [
    "initialize_projector",
    "get_batch_opus",
    "compute_GradProd_GC_per_iter",
    "find_GClayers",
    "greedy_selection",
    "stochastic_greedy_selection",
    "GradientProjector",
]
