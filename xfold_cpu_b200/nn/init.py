"""Deterministic random initialisation used by the benchmarks and tests.

The reference's benchmark configs use random-init weights: every Linear
weight and bias, and the other plain parameters (OuterProductMean's output_w
and output_b), ~ N(0, std) with std = 0.02; LayerNorm gamma = 1, beta = 0.
`perturb_layer_norm` draws gamma ~ 1 + 0.1 N(0,1), beta ~ 0.1 N(0,1) instead,
so tests exercise the affine path.  Parameters are drawn on the CPU from one
torch.Generator in named_parameters() order (reproducible on any machine).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..fastnn import LayerNorm


@torch.no_grad()
def init_params_(module: nn.Module, seed: int = 0, std: float = 0.02,
                 perturb_layer_norm: bool = False) -> nn.Module:
    g = torch.Generator().manual_seed(seed)
    for name, p in module.named_parameters():
        leaf = name.rsplit(".", 1)[-1]
        owner = module.get_submodule(name.rsplit(".", 1)[0]) if "." in name else module
        is_norm = isinstance(owner, (LayerNorm, nn.LayerNorm))
        if is_norm:
            if perturb_layer_norm:
                v = torch.randn(p.shape, generator=g) * 0.1
                v = v + 1.0 if leaf == "weight" else v
            else:
                v = torch.ones(p.shape) if leaf == "weight" else torch.zeros(p.shape)
        else:
            v = torch.randn(p.shape, generator=g) * std
        p.copy_(v.to(p.dtype))
    return module
