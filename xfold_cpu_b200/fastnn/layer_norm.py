"""fastnn.LayerNorm with the `cuda` implementation (xfold/fastnn/layer_norm.py:14-87).

Same constructor, parameters (weight / bias, γ=1 β=0 at init) and eps.  The
forward returns bf16 — the dtype the next autocast linear consumes."""

from __future__ import annotations

import numbers

import torch
import torch.nn as nn

from .. import native
from . import config


class LayerNorm(nn.Module):
    def __init__(self, normalized_shape, eps: float = 1e-5, elementwise_affine: bool = True,
                 bias: bool = True, device=None, dtype=None) -> None:
        super().__init__()
        if isinstance(normalized_shape, numbers.Integral):
            normalized_shape = (normalized_shape,)
        self.normalized_shape = tuple(normalized_shape)
        self.eps = eps
        self.elementwise_affine = elementwise_affine
        kw = {"device": device, "dtype": dtype}
        if elementwise_affine:
            self.weight = nn.Parameter(torch.empty(self.normalized_shape, **kw))
            if bias:
                self.bias = nn.Parameter(torch.empty(self.normalized_shape, **kw))
            else:
                self.register_parameter("bias", None)
        else:
            self.register_parameter("weight", None)
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        if self.elementwise_affine:
            nn.init.ones_(self.weight)
            if self.bias is not None:
                nn.init.zeros_(self.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        config.require_cuda("layer_norm_implementation")
        if len(self.normalized_shape) != 1:
            raise ValueError("the cuda LayerNorm normalises over the last dimension only")
        return native.layer_norm(x, self.weight, self.bias, self.eps)

    def extra_repr(self) -> str:
        return f"{self.normalized_shape}, eps={self.eps}, elementwise_affine={self.elementwise_affine}"
