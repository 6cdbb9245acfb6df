"""fastnn.gated_linear_unit with the `cuda` implementation
(xfold/fastnn/gated_linear_unit.py:103-122)."""

from __future__ import annotations

import torch

from .. import native
from . import config
from .weight_cache import WeightCache


def _pack(weight_kn: torch.Tensor) -> torch.Tensor:
    return native.pack_glu_weight(weight_kn.T)


def gated_linear_unit(x: torch.Tensor, weight: torch.Tensor,
                      weight_cache: WeightCache | None = None) -> torch.Tensor:
    """silu(a) * b with a, b = chunk(x @ weight, 2).  `weight` is [K, 2N] as in the
    reference (transition1.weight.T); the cache keeps its packed bf16 copy."""
    config.require_cuda("gated_linear_unit_implementation")
    packed = weight_cache.get((weight,), _pack) if weight_cache is not None else _pack(weight)
    return native.gated_linear_unit(x, packed, weight_packed=True)
