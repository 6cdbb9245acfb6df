"""fastnn.dot_product_attention with the `cuda` implementation
(dispatcher xfold/fastnn/attention.py:69-98, semantics of the torch path :45-66)."""

from __future__ import annotations

import torch

from .. import native
from . import config


def dot_product_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          mask: torch.Tensor | None = None, bias: torch.Tensor | None = None):
    """softmax(q k^T * d^-0.5 + bias, masked -> -1e9) v; 3-D inputs get a batch
    dimension as in the reference dispatcher."""
    config.require_cuda("dot_product_attention_implementation")
    squeeze = q.dim() == 3
    if squeeze:
        q, k, v = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0)
    out = native.dot_product_attention(q, k, v, mask=mask, bias=bias)
    return out.squeeze(0) if squeeze else out
