"""Row-sharded Pairformer block: the pair split by rows over GPUs.

The reference runs every pair operator on the whole N x N pair inside one
process (xfold/nn/pairformer.py:77-114).  Here rank r of G holds pair rows
R_r = [r N/G, (r+1) N/G) as a [N/G, N, c] f32 block and the operators run on
row blocks through the library's row-block stages, with exchanges only where
the arithmetic crosses rows:

* Triangle multiplication (both directions): the projection is row-local; an
  all-to-all turns the row blocks of a, b [c, N/G, N] into channel shards
  [c/G, N, N]; each rank contracts its channels over the whole pair; a second
  all-to-all returns the rows of every channel for the centre LayerNorm and the
  gated output projection, which add into the local rows.
* Grid attention, starting node: LayerNorm and the bias rows are row-local; the
  bias [heads, N, N] is all-gathered; attention runs on the local rows.
* Grid attention, ending node: the same bias all-gather, plus an all-to-all
  transpose of the LayerNorm'd pair (rank r receives columns R_r), attention
  over those columns with the un-transposed mask rows of the same indices (as
  the reference, attention.py:99-100), and the transpose back of the update.
* Transition: row-local.
* Single track: the pair-logit rows are all-gathered; the single representation
  (N x 384) is replicated and every process updates its own copy identically.

Exchanges go through an `Exchange`: `ProcessGroupExchange` (one shard per
process over torch.distributed -- NCCL over NVLink on GPUs, gloo on CPU) or
`LocalExchange` (all shards in one process, for checking the sharded arithmetic
on one device).  Exchanges copy whole tensors into this GPU's memory; no kernel
reads another GPU's memory.

The compute of each stage comes from a `stages` object; `NativeStages` (the
CUDA kernels) is the default and the only one this package provides.
"""

from __future__ import annotations

from typing import Protocol

import torch

from . import native
from .nn.modules import (GridSelfAttention, PairformerBlock, TriangleMultiplication, _bf16)


# ----------------------------------------------------------------------------- exchanges

class Exchange(Protocol):
    world: int
    ranks: list[int]  # global rank of each local shard

    def all_to_all(self, bufs: list[torch.Tensor]) -> list[torch.Tensor]:
        """bufs[l] is [G, ...] (chunk s goes to rank s); returns [G, ...] per
        local shard (chunk t came from rank t)."""

    def all_gather(self, bufs: list[torch.Tensor]) -> list[torch.Tensor]:
        """bufs[l] is [...]; returns [G, ...] per local shard (rank t's tensor at t)."""


class ProcessGroupExchange:
    """One shard per process over torch.distributed (NCCL or gloo)."""

    def __init__(self, group=None) -> None:
        import torch.distributed as dist

        self._dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.ranks = [dist.get_rank(group)]

    def all_to_all(self, bufs):
        (buf,) = bufs
        out = torch.empty_like(buf)
        self._dist.all_to_all_single(out, buf.contiguous(), group=self.group)
        return [out]

    def all_gather(self, bufs):
        (buf,) = bufs
        buf = buf.contiguous()
        out = torch.empty((self.world * buf.shape[0], *buf.shape[1:]), dtype=buf.dtype,
                          device=buf.device)
        self._dist.all_gather_into_tensor(out, buf, group=self.group)
        return [out.view(self.world, *buf.shape)]


class LocalExchange:
    """All G shards in this process (tensor copies stand in for the transfers)."""

    def __init__(self, world: int) -> None:
        self.world = world
        self.ranks = list(range(world))

    def all_to_all(self, bufs):
        g = self.world
        return [torch.stack([bufs[t][r] for t in range(g)]) for r in range(g)]

    def all_gather(self, bufs):
        stacked = torch.stack(list(bufs))
        return [stacked.clone() for _ in range(self.world)]


# ----------------------------------------------------------------------------- stages

class NativeStages:
    """Row-block stages on the CUDA kernels, using each module's cached weights."""

    def trimul_project(self, mod: TriangleMultiplication, pair_rows, mask_rows):
        packed = mod._packed.get(
            (mod.projection.weight, mod.gate.weight, mod.gating_linear.weight),
            native.pack_triangle_weights)
        return native.triangle_projection(pair_rows, mask_rows, mod.left_norm_input.weight,
                                          mod.left_norm_input.bias, mod.left_norm_input.eps,
                                          packed)

    def trimul_contract(self, mod: TriangleMultiplication, a, b):
        return native.triangle_contraction(a, b, mod.outgoing)

    def trimul_output(self, mod: TriangleMultiplication, z_rows, g, pair_rows):
        native.triangle_output(z_rows, g, mod.center_norm.weight, mod.center_norm.bias,
                               mod.center_norm.eps, _bf16(mod._out_w, mod.output_projection.weight),
                               out=pair_rows, accumulate=True)

    def attention_prepare(self, mod: GridSelfAttention, pair_rows):
        return native.grid_attention_prepare(pair_rows, mod.act_norm.weight, mod.act_norm.bias,
                                             mod.act_norm.eps,
                                             _bf16(mod._bias_w, mod.pair_bias_projection.weight),
                                             mod.num_head)

    def attention_rows(self, mod: GridSelfAttention, x_rows, mask_rows, bias, out=None):
        packed = mod._packed.get(
            (mod.q_projection.weight, mod.k_projection.weight, mod.v_projection.weight,
             mod.gating_query.weight), native.pack_attention_weights)
        ow = _bf16(mod._out_w, mod.output_projection.weight)
        if out is None:
            return native.grid_attention_rows(x_rows, mask_rows, bias, packed, ow, mod.num_head)
        return native.grid_attention_rows(x_rows, mask_rows, bias, packed, ow, mod.num_head,
                                          out=out, accumulate=True)

    def transition(self, block: PairformerBlock, pair_rows):
        block.pair_transition.accumulate_(pair_rows)

    def pair_logits_rows(self, block: PairformerBlock, pair_rows):
        norm = block.single_pair_logits_norm
        return native.pair_logits_rows(pair_rows, norm.weight, norm.bias, norm.eps,
                                       _bf16(block._logits_w, block.single_pair_logits_projection.weight))

    def single_track(self, block: PairformerBlock, single, seq_mask, logits):
        block.single_attention_.accumulate_(single, seq_mask, logits)
        block.single_transition.accumulate_(single)


# ----------------------------------------------------------------------------- the block

def shard_rows(n: int, world: int, rank: int) -> slice:
    """Rows of rank `rank`: an even split (n % world == 0)."""
    per = n // world
    return slice(rank * per, (rank + 1) * per)


def check_sharding(n: int, c: int, world: int) -> None:
    if world < 1 or n % world or c % world:
        raise ValueError(f"a row-sharded pair needs N ({n}) and c ({c}) divisible by the "
                         f"number of ranks ({world})")
    if n % 8:
        raise ValueError("a row-sharded pair needs N % 8 == 0")


def _triangle(mod, pairs, pair_mask, exchange, stages):
    g = exchange.world
    rows, n, c = pairs[0].shape
    cs = c // g
    a_list, b_list, g_list = [], [], []
    for pair, r in zip(pairs, exchange.ranks):
        a, b, gate = stages.trimul_project(mod, pair, pair_mask[shard_rows(n, g, r)])
        a_list.append(a.view(g, cs, rows, n))  # chunk s = channels of rank s
        b_list.append(b.view(g, cs, rows, n))
        g_list.append(gate)
    a_recv = exchange.all_to_all(a_list)  # [t, cs, rows of t, n]
    b_recv = exchange.all_to_all(b_list)
    del a_list, b_list
    z_send = []
    for ar, br in zip(a_recv, b_recv):
        a_full = ar.transpose(0, 1).reshape(cs, n, n)
        b_full = br.transpose(0, 1).reshape(cs, n, n)
        z = stages.trimul_contract(mod, a_full, b_full)  # [cs, n, n], my channels, all rows
        z_send.append(z.view(cs, g, rows, n).transpose(0, 1).contiguous())  # chunk s = rows of s
    del a_recv, b_recv
    z_recv = exchange.all_to_all(z_send)  # [t, cs (channels of t), my rows, n]
    for pair, zr, gate in zip(pairs, z_recv, g_list):
        stages.trimul_output(mod, zr.view(c, rows, n), gate, pair)


def _bias_full(bias_rows, exchange):
    gathered = exchange.all_gather(bias_rows)  # [G, heads, rows, n]
    return [t.transpose(0, 1).reshape(t.shape[1], -1, t.shape[-1]) for t in gathered]


def _transpose_blocks(blocks, exchange):
    """Row blocks [rows, n, ...] -> the matching column blocks [rows (columns of
    this rank), n (all rows), ...] through one all-to-all."""
    g = exchange.world
    sends = []
    for x in blocks:
        rows, n = x.shape[:2]
        sends.append(x.view(rows, g, rows, *x.shape[2:]).transpose(0, 1).contiguous())
    recv = exchange.all_to_all(sends)  # [t, rows of t (i), my columns (j), ...]
    out = []
    for t in recv:
        g_, rows, cols = t.shape[:3]
        out.append(t.permute(2, 0, 1, *range(3, t.dim())).reshape(cols, g_ * rows, *t.shape[3:]))
    return out


def _attention(mod, pairs, pair_mask, exchange, stages):
    g = exchange.world
    rows, n, _ = pairs[0].shape
    prepared = [stages.attention_prepare(mod, pair) for pair in pairs]
    biases = _bias_full([bias for _, bias in prepared], exchange)
    if not mod.transpose:
        for pair, (x, _), bias, r in zip(pairs, prepared, biases, exchange.ranks):
            stages.attention_rows(mod, x, pair_mask[shard_rows(n, g, r)], bias, out=pair)
        return
    # ending node: attention runs over pair columns; mask rows indexed by the column
    cols = _transpose_blocks([x for x, _ in prepared], exchange)
    del prepared
    updates = [stages.attention_rows(mod, xt, pair_mask[shard_rows(n, g, r)], bias)
               for xt, bias, r in zip(cols, biases, exchange.ranks)]
    for pair, upd in zip(pairs, _transpose_blocks(updates, exchange)):
        pair += upd


def pairformer_block(block: PairformerBlock, pairs: list[torch.Tensor], pair_mask: torch.Tensor,
                     single: torch.Tensor | None, seq_mask: torch.Tensor | None,
                     exchange: Exchange, stages=None):
    """One Pairformer block on a row-sharded pair, updated in place.

    pairs: this process's row blocks ([N/G, N, c] f32 contiguous, one per local
    shard, in `exchange.ranks` order); pair_mask: the full [N, N] mask (every
    process holds it); single / seq_mask: this process's copy of the single
    track, updated in place (once per process)."""
    stages = NativeStages() if stages is None else stages
    rows, n, c = pairs[0].shape
    check_sharding(n, c, exchange.world)
    if rows * exchange.world != n:
        raise ValueError("each shard must hold N / world rows")
    _triangle(block.triangle_multiplication_outgoing, pairs, pair_mask, exchange, stages)
    _triangle(block.triangle_multiplication_incoming, pairs, pair_mask, exchange, stages)
    _attention(block.pair_attention1, pairs, pair_mask, exchange, stages)
    _attention(block.pair_attention2, pairs, pair_mask, exchange, stages)
    for pair in pairs:
        stages.transition(block, pair)
    if not block.with_single:
        return pairs
    logits = _bias_full([stages.pair_logits_rows(block, pair) for pair in pairs], exchange)
    stages.single_track(block, single, seq_mask, logits[0])
    return pairs, single
