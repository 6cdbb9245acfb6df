"""xfold hot-path modules with the `cuda` backend (same names and parameters
as xfold.nn)."""

from .modules import (AdaLNZero, AdaptiveLayerNorm, CrossAttention, DiffusionCrossAttTransformer,
                      DiffusionTransformer, DiffusionTransition, EvoformerBlock, GridSelfAttention,
                      MSAAttention, OuterProductMean, PairformerBlock, SelfAttention, Transition,
                      TriangleMultiplication)
from .atom_layout import GatherInfo
from .init import init_params_

__all__ = ["AdaLNZero", "AdaptiveLayerNorm", "CrossAttention", "DiffusionCrossAttTransformer",
           "DiffusionTransformer", "DiffusionTransition", "EvoformerBlock", "GatherInfo",
           "MSAAttention", "OuterProductMean",
           "GridSelfAttention", "PairformerBlock", "SelfAttention", "Transition",
           "TriangleMultiplication", "init_params_"]
