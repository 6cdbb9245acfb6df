"""xfold hot-path modules with the `cuda` backend (same names and parameters
as xfold.nn)."""

from .modules import (AdaLNZero, AdaptiveLayerNorm, DiffusionTransformer, DiffusionTransition,
                      GridSelfAttention, PairformerBlock, SelfAttention, Transition,
                      TriangleMultiplication)
from .init import init_params_

__all__ = ["AdaLNZero", "AdaptiveLayerNorm", "DiffusionTransformer", "DiffusionTransition",
           "GridSelfAttention", "PairformerBlock", "SelfAttention", "Transition",
           "TriangleMultiplication", "init_params_"]
