"""xfold hot-path modules with the `cuda` backend (same names and parameters
as xfold.nn)."""

from .modules import (AdaLNZero, AdaptiveLayerNorm, CrossAttention, DiffusionCrossAttTransformer,
                      DiffusionTransformer, DiffusionTransition, GridSelfAttention,
                      PairformerBlock, SelfAttention, Transition, TriangleMultiplication)
from .atom_layout import GatherInfo
from .init import init_params_

__all__ = ["AdaLNZero", "AdaptiveLayerNorm", "CrossAttention", "DiffusionCrossAttTransformer",
           "DiffusionTransformer", "DiffusionTransition", "GatherInfo",
           "GridSelfAttention", "PairformerBlock", "SelfAttention", "Transition",
           "TriangleMultiplication", "init_params_"]
