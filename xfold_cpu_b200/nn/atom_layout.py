"""Atom-layout gather description used by the atom transformer.

GatherInfo mirrors xfold/nn/atom_layout.py:20-86 (the same fields, so a
featurised batch's `queries_to_keys` passes through unchanged), and convert()
restates xfold/nn/atom_layout.py:88-160: the layout axes are flattened, rows
are gathered by `gather_idxs` and rows whose `gather_mask` is False are zeroed.
DiffusionCrossAttTransformer does not call convert() on its hot path: the
gather of the keys is fused into the keys' LayerNorm kernel, which reads the
index and mask directly (`key_gather`).
"""

from __future__ import annotations

import dataclasses
from typing import Any

import torch


@dataclasses.dataclass(frozen=True)
class GatherInfo:
    gather_idxs: torch.Tensor
    gather_mask: torch.Tensor
    input_shape: torch.Tensor

    def __post_init__(self):
        if self.gather_mask.shape != self.gather_idxs.shape:
            raise ValueError(
                "All arrays must have the same shape. Got\n"
                f"gather_idxs.shape = {self.gather_idxs.shape}\n"
                f"gather_mask.shape = {self.gather_mask.shape}\n")

    def __getitem__(self, key: Any) -> "GatherInfo":
        return GatherInfo(self.gather_idxs[key], self.gather_mask[key], self.input_shape)

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self.gather_idxs.shape)


def convert(gather_info: GatherInfo, arr: torch.Tensor, *,
            layout_axes: tuple[int, ...] = (0,)) -> torch.Tensor:
    """arr with its layout axes replaced by gather_info's shape."""
    layout_axes = tuple(i if i >= 0 else i + arr.ndim for i in layout_axes)
    begin, end = layout_axes[0], layout_axes[-1] + 1
    if layout_axes != tuple(range(begin, end)):
        raise ValueError(f"layout_axes must be continuous. Got {layout_axes}.")
    layout_shape = arr.shape[begin:end]
    input_shape = [int(v) for v in torch.as_tensor(gather_info.input_shape).flatten()]
    if len(layout_shape) != len(input_shape) or layout_shape[0] < input_shape[0] or \
            list(layout_shape[1:]) != input_shape[1:]:
        raise ValueError(
            f"Input array layout axes are incompatible. You specified layout axes {layout_axes} "
            f"with an input array of shape {tuple(arr.shape)}, but the gather info expects "
            f"shape {tuple(input_shape)}.")
    flat = arr.reshape(arr.shape[:begin] + (-1,) + arr.shape[end:])
    index = (slice(None),) * begin + (gather_info.gather_idxs.to(arr.device),)
    out = flat[index]
    mask_shape = (1,) * begin + tuple(gather_info.gather_mask.shape) + (1,) * (arr.ndim - end)
    return out * gather_info.gather_mask.to(arr.device).reshape(mask_shape)


def key_gather(gather_info: GatherInfo, source_rows: int,
               device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """(index int64, valid bool) on `device` for the fused gather: indices
    checked against the flattened source like torch indexing (IndexError), and
    negative ones wrapped."""
    idx = gather_info.gather_idxs.to(device=device, dtype=torch.int64)
    if idx.numel() and (bool((idx < -source_rows).any()) or bool((idx >= source_rows).any())):
        raise IndexError(f"gather index out of range for {source_rows} source rows")
    idx = torch.where(idx < 0, idx + source_rows, idx).contiguous()
    valid = gather_info.gather_mask.to(device=device, dtype=torch.bool).contiguous()
    return idx, valid
