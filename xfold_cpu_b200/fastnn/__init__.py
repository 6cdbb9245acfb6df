"""`cuda` implementations of xfold.fastnn (LayerNorm, dot_product_attention,
gated_linear_unit), mirroring xfold/fastnn/__init__.py:1-5."""

from .layer_norm import LayerNorm
from .attention import dot_product_attention
from .gated_linear_unit import gated_linear_unit
from .weight_cache import WeightCache
from . import config

__all__ = ["LayerNorm", "dot_product_attention", "gated_linear_unit", "WeightCache", "config"]
