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
* Single track: sharded by query rows.  A rank's pair-logit rows are the bias
  rows of its own queries, so each rank attends for its rows against every key
  (LayerNorm and projections of all N tokens are repeated on every rank, which
  is cheap), runs the single transition on them, and the updated rows of the
  single representation (N x 384 f32) are all-gathered.

Routed stages: where the exchange class supports it (`routes`) and the stages
do (`NativeStages`), the producer of each exchanged tensor stores it straight
into the receive buffers of the ranks that need it -- the TriMul projection
writes a and b by channel owner, the contraction writes z rows by row owner,
the ending node's LayerNorm writes the transposed rows and its output
projection the transposed update -- and a barrier follows, so no separate copy
runs.

Exchanges go through one of three classes with the same four patterns:
`PeerExchange` (one shard per GPU: the library's copy kernel stores each chunk
straight into the peers' receive buffers over NVLink, then a flag barrier --
release stores of an epoch into every GPU's flag array and a bounded wait -- or
a one-element NCCL all-reduce), `ProcessGroupExchange` (one shard per process over
torch.distributed all-to-all / all-gather -- NCCL on GPUs, gloo on CPU) and
`LocalExchange` (all shards in one process, for checking the sharded arithmetic
on one device).  No kernel reads another GPU's memory: peer traffic is stores
only, and no TMA or multicast is involved.

The compute of each stage comes from a `stages` object; `NativeStages` (the
CUDA kernels) is the default and the only one this package provides.
"""

from __future__ import annotations

import torch

from . import native
from .nn.modules import (GridSelfAttention, PairformerBlock, TriangleMultiplication, _bf16)


# ----------------------------------------------------------------------------- exchanges
# An exchange moves row-sharded data between the G ranks.  The driver needs four
# patterns; each takes one tensor per local shard (in `ranks` order) and returns
# one per local shard:
#   rows_to_channels   [c, rows, n]  -> [c/G, n, n]   (rows of every rank, my channels)
#   channels_to_rows   [c/G, n, n]   -> [c, rows, n]  (channels of every rank, my rows)
#   gather_rows        [h, rows, n]  -> [h, n, n]     (every rank's rows)
#   transpose          [rows, n, c]  -> [rows, n, c]  (x[i, j] -> y[j, i]: my columns, all rows)


class CollectiveExchange:
    """The four patterns from all-to-all / all-gather primitives plus tensor
    permutes.  Subclasses provide `world`, `ranks`, `all_to_all` (bufs[l] is
    [G, ...], chunk s for rank s; returns [G, ...], chunk t from rank t) and
    `all_gather` (returns [G, ...], rank t's tensor at t)."""

    world: int
    ranks: list[int]

    def rows_to_channels(self, blocks):
        g = self.world
        c, rows, n = blocks[0].shape
        recv = self.all_to_all([t.view(g, c // g, rows, n) for t in blocks])
        return [t.transpose(0, 1).reshape(c // g, g * rows, n) for t in recv]

    def rows_to_channels_pair(self, a_blocks, b_blocks):
        """rows_to_channels of the TriMul operands a and b."""
        return self.rows_to_channels(a_blocks), self.rows_to_channels(b_blocks)

    def channels_to_rows(self, blocks):
        g = self.world
        cs, n, _ = blocks[0].shape
        rows = n // g
        sends = [t.view(cs, g, rows, n).transpose(0, 1).contiguous() for t in blocks]
        return [t.view(g * cs, rows, n) for t in self.all_to_all(sends)]

    def gather_rows(self, blocks):
        gathered = self.all_gather(blocks)
        return [t.transpose(0, 1).reshape(t.shape[1], -1, t.shape[-1]) for t in gathered]

    def transpose(self, blocks):
        g = self.world
        sends = []
        for x in blocks:
            rows = x.shape[0]
            sends.append(x.view(rows, g, rows, *x.shape[2:]).transpose(0, 1).contiguous())
        out = []
        for t in self.all_to_all(sends):  # [t, rows of t (i), my columns (j), ...]
            g_, rows, cols = t.shape[:3]
            out.append(t.permute(2, 0, 1, *range(3, t.dim())).reshape(cols, g_ * rows, *t.shape[3:]))
        return out


class ProcessGroupExchange(CollectiveExchange):
    """One shard per process over torch.distributed collectives (NCCL or gloo)."""

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


class LocalExchange(CollectiveExchange):
    """All G shards in this process (tensor copies stand in for the transfers).
    With routed=True (CUDA tensors) the routed stages store into G receive
    buffers on this device, as they would into G GPUs' buffers."""

    def __init__(self, world: int, routed: bool = False) -> None:
        self.world = world
        self.ranks = list(range(world))
        self.routes = routed

    def route(self, kind, shape, dtype, device):
        bufs = [torch.empty(shape, dtype=dtype, device=device) for _ in range(self.world)]
        ptrs = [b.data_ptr() for b in bufs]
        return [(bufs[r], native.Route(ptrs, r)) for r in range(self.world)]

    def complete(self, device):
        pass  # one stream: the stores are in order

    def all_to_all(self, bufs):
        g = self.world
        return [torch.stack([bufs[t][r] for t in range(g)]) for r in range(g)]

    def all_gather(self, bufs):
        stacked = torch.stack(list(bufs))
        return [stacked.clone() for _ in range(self.world)]


class PeerExchange:
    """One shard per GPU; each pattern is one launch of the library's exchange
    copy kernel that stores straight into the peers' receive buffers over NVLink
    (mapped into this process by CUDA IPC), each chunk at its final position, so
    no permute copies are needed on either side.  After the copy comes a
    barrier: by default the library's flag barrier (each GPU writes an epoch
    into a flag slot on every GPU with system-scope release stores, then waits,
    bounded, until its own slots hold it); with barrier="nccl" (or
    XFB_EXCHANGE_BARRIER=nccl) a one-element NCCL all-reduce.  When the barrier
    completes on a rank, every rank's stores into that rank's buffer have
    landed.  Receive buffers alternate between two copies per pattern, so the
    barrier after an exchange also guarantees that nobody still reads the copy
    the next exchange overwrites (every consumer of a buffer is enqueued before
    its rank's next barrier).
    The returned tensors are views of those buffers: valid until the same
    pattern with the same shape has run twice more."""

    def __init__(self, group=None, barrier: str | None = None, routed: bool | None = None) -> None:
        import os

        import torch.distributed as dist

        # routed stages (producers store straight into the peers' buffers) unless
        # routed=False or XFB_EXCHANGE_ROUTED=0
        self.routes = (os.environ.get("XFB_EXCHANGE_ROUTED", "1") != "0"
                       if routed is None else bool(routed))
        self._dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.ranks = [self.rank]
        self._bufs: dict = {}
        self._flag = None
        self.barrier = barrier or os.environ.get("XFB_EXCHANGE_BARRIER", "flags")
        if self.barrier not in ("flags", "nccl"):
            raise ValueError("barrier must be 'flags' or 'nccl'")
        self._flags = None  # (local flag array, every GPU's array, epoch counter)

    # -- receive buffers, shared once per (pattern, shape, dtype)
    def _recv(self, kind, shape, dtype, device):
        key = (kind, tuple(shape), dtype)
        entry = self._bufs.get(key)
        if entry is None:
            copies = []
            for _ in range(2):
                local = torch.empty(shape, dtype=dtype, device=device)
                metas = [None] * self.world
                self._dist.all_gather_object(metas, _ipc_handle(local), group=self.group)
                peers = [local.data_ptr() if r == self.rank else _ipc_open(*meta)
                         for r, meta in enumerate(metas)]
                copies.append((local, peers))
            entry = {"copies": copies, "next": 0}
            self._bufs[key] = entry
        local, peers = entry["copies"][entry["next"]]
        entry["next"] ^= 1
        return local, peers

    # -- routed stages: the producing kernels store into the receive buffers
    def route(self, kind, shape, dtype, device):
        """[(this rank's next receive buffer of `kind`, the route to every rank's
        copy of it)] for a routed stage; complete() (or the next exchange's
        barrier) publishes what the stage stored."""
        local, peers = self._recv(kind, shape, dtype, device)
        return [(local, native.Route(peers, self.rank))]

    def complete(self, device):
        """The exchange barrier after routed stores."""
        self._sync(device)

    def _copy_and_sync(self, boxes, device):
        import ctypes

        from . import _capi

        stream = torch.cuda.current_stream(device).cuda_stream
        arr = (_capi.CopyBox * len(boxes))(*boxes)
        _capi.call("xfb_exchange_copy", ctypes_addressof(arr), len(boxes), stream)
        self._sync(device)

    def _sync(self, device):
        import ctypes

        from . import _capi

        stream = torch.cuda.current_stream(device).cuda_stream
        if self.barrier == "nccl":
            if self._flag is None:
                self._flag = torch.zeros(1, dtype=torch.int32, device=device)
            self._dist.all_reduce(self._flag, group=self.group)
            return
        if self._flags is None:
            local = torch.zeros(16, dtype=torch.int32, device=device)
            metas = [None] * self.world
            self._dist.all_gather_object(metas, _ipc_handle(local), group=self.group)
            ptrs = [local.data_ptr() if r == self.rank else _ipc_open(*meta)
                    for r, meta in enumerate(metas)]
            torch.cuda.synchronize(device)  # the zero fill is done before any peer signals
            self._dist.barrier(group=self.group)
            # the epoch lives on the device (advanced by each signal), so a
            # captured CUDA graph of exchanges can be replayed
            counter = torch.zeros(1, dtype=torch.int32, device=device)
            self._flags = (local, (ctypes.c_void_p * self.world)(*ptrs), counter)
        local, peers, counter = self._flags
        _capi.call("xfb_exchange_signal_counted", ctypes_addressof(peers), self.world, self.rank,
                   counter.data_ptr(), stream)
        _capi.call("xfb_exchange_wait_counted", local.data_ptr(), self.world, counter.data_ptr(),
                   stream)

    def _box(self, src_ptr, dst_ptr, d0, d1, d2_bytes, s0, s1, t0, t1):
        from . import _capi

        return _capi.CopyBox(src_ptr, dst_ptr, d0, d1, d2_bytes, s0, s1, t0, t1)

    def _r2c_boxes(self, a, kind):
        g, r = self.world, self.rank
        c, rows, n = a.shape
        cs, e = c // g, a.element_size()
        local, peers = self._recv(kind, (cs, n, n), a.dtype, a.device)
        boxes = [self._box(a.data_ptr() + s * cs * rows * n * e, peers[s] + r * rows * n * e,
                           cs, rows, n * e, rows * n * e, n * e, n * n * e, n * e)
                 for s in range(g)]
        return local, boxes

    def rows_to_channels(self, blocks):
        (a,) = blocks
        a = a.contiguous()
        local, boxes = self._r2c_boxes(a, "r2c")
        self._copy_and_sync(boxes, a.device)
        return [local]

    def rows_to_channels_pair(self, a_blocks, b_blocks):
        """rows_to_channels of a and b in one copy launch and one barrier."""
        (a,), (b,) = a_blocks, b_blocks
        a, b = a.contiguous(), b.contiguous()
        la, boxes_a = self._r2c_boxes(a, "r2c")
        lb, boxes_b = self._r2c_boxes(b, "r2c_b")
        self._copy_and_sync(boxes_a + boxes_b, a.device)
        return [la], [lb]

    def channels_to_rows(self, blocks):
        (z,) = blocks
        g, r = self.world, self.rank
        z = z.contiguous()
        cs, n, _ = z.shape
        rows, e = n // g, z.element_size()
        local, peers = self._recv("c2r", (g * cs, rows, n), z.dtype, z.device)
        boxes = [self._box(z.data_ptr() + s * rows * n * e, peers[s] + r * cs * rows * n * e,
                           cs, rows, n * e, n * n * e, n * e, rows * n * e, n * e)
                 for s in range(g)]
        self._copy_and_sync(boxes, z.device)
        return [local]

    def gather_rows(self, blocks):
        (t,) = blocks
        g, r = self.world, self.rank
        t = t.contiguous()
        h, rows, n = t.shape
        e = t.element_size()
        local, peers = self._recv("gather", (h, g * rows, n), t.dtype, t.device)
        boxes = [self._box(t.data_ptr(), peers[s] + r * rows * n * e,
                           h, rows, n * e, rows * n * e, n * e, g * rows * n * e, n * e)
                 for s in range(g)]
        self._copy_and_sync(boxes, t.device)
        return [local]

    def transpose(self, blocks):
        (x,) = blocks
        g, r = self.world, self.rank
        x = x.contiguous()
        rows, n, c = x.shape
        e = x.element_size()
        local, peers = self._recv("transpose", (rows, n, c), x.dtype, x.device)
        # x[ii, s*rows + jj, :] -> rank s's y[jj, r*rows + ii, :]
        boxes = [self._box(x.data_ptr() + s * rows * c * e, peers[s] + r * rows * c * e,
                           rows, rows, c * e, n * c * e, c * e, c * e, n * c * e)
                 for s in range(g)]
        self._copy_and_sync(boxes, x.device)
        return [local]


# PeerExchange, ProcessGroupExchange and LocalExchange share the four patterns
# above (plus `world` and `ranks`), which is all pairformer_block uses.


def _ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """IPC handle of the allocation holding t, and t's byte offset in it."""
    import ctypes

    from . import _capi

    lib = _capi.load()
    buf = ctypes.create_string_buffer(int(lib.xfb_ipc_handle_bytes()))
    off = ctypes.c_int64(0)
    _capi.call("xfb_ipc_handle", t.data_ptr(), buf, ctypes.byref(off))
    return buf.raw, off.value


def _ipc_open(handle: bytes, offset: int) -> int:
    """Maps a peer's allocation on the current device; the address of its tensor."""
    import ctypes

    from . import _capi

    ptr = ctypes.c_void_p(0)
    _capi.call("xfb_ipc_open", ctypes.create_string_buffer(handle, len(handle)), offset,
               ctypes.byref(ptr))
    return int(ptr.value)


def ctypes_addressof(arr) -> int:
    import ctypes

    return ctypes.addressof(arr)


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

    def single_attention_rows(self, block: PairformerBlock, x, seq_mask, logits_rows, row0, out):
        att = block.single_attention_
        packed = att._packed.get(
            (att.q_projection.weight, att.k_projection.weight, att.v_projection.weight,
             att.gating_query.weight), native.pack_attention_weights)
        ln = att.adaptive_layernorm.layer_norm
        native.self_attention_rows(x, seq_mask, logits_rows, row0, ln.weight, ln.bias, ln.eps,
                                   packed, att.q_projection.bias,
                                   _bf16(att._wo, att.adaptive_zero_init.transition2.weight),
                                   att.num_head, out, accumulate=True)

    def single_transition_rows(self, block: PairformerBlock, single_rows):
        block.single_transition.accumulate_(single_rows)

    # -- routed forms (the exchange after the stage done by its kernel)
    routed = True

    def trimul_project_routed(self, mod: TriangleMultiplication, pair_rows, mask_rows, a_route,
                              b_route):
        packed = mod._packed.get(
            (mod.projection.weight, mod.gate.weight, mod.gating_linear.weight),
            native.pack_triangle_weights)
        return native.triangle_projection_routed(pair_rows, mask_rows, mod.left_norm_input.weight,
                                                 mod.left_norm_input.bias,
                                                 mod.left_norm_input.eps, packed, a_route, b_route)

    def trimul_contract_routed(self, mod: TriangleMultiplication, a, b, z_route):
        native.triangle_contraction_routed(a, b, mod.outgoing, z_route)

    def attention_prepare_routed(self, mod: GridSelfAttention, pair_rows, x_route):
        return native.grid_attention_prepare_routed(
            pair_rows, mod.act_norm.weight, mod.act_norm.bias, mod.act_norm.eps,
            _bf16(mod._bias_w, mod.pair_bias_projection.weight), mod.num_head, x_route)

    def attention_rows_routed(self, mod: GridSelfAttention, x_rows, mask_rows, bias, out_route):
        packed = mod._packed.get(
            (mod.q_projection.weight, mod.k_projection.weight, mod.v_projection.weight,
             mod.gating_query.weight), native.pack_attention_weights)
        native.grid_attention_rows_routed(x_rows, mask_rows, bias, packed,
                                          _bf16(mod._out_w, mod.output_projection.weight),
                                          mod.num_head, out_route)


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


def _routed(exchange, stages) -> bool:
    return bool(getattr(exchange, "routes", False) and getattr(stages, "routed", False))


def _triangle(mod, pairs, pair_mask, exchange, stages):
    g = exchange.world
    rows, n, c = pairs[0].shape
    if _routed(exchange, stages):
        dev = pairs[0].device
        # projection -> (rows -> channels) -> contraction -> (channels -> rows),
        # each exchange stored by its producer, then one barrier
        ra = exchange.route("r2c", (c // g, n, n), torch.bfloat16, dev)
        rb = exchange.route("r2c_b", (c // g, n, n), torch.bfloat16, dev)
        gates = [stages.trimul_project_routed(mod, pair, pair_mask[shard_rows(n, g, r)], ta, tb)
                 for pair, r, (_, ta), (_, tb) in zip(pairs, exchange.ranks, ra, rb)]
        exchange.complete(dev)
        rz = exchange.route("c2r", (c, rows, n), torch.bfloat16, dev)
        for (a, _), (b, _), (_, tz) in zip(ra, rb, rz):
            stages.trimul_contract_routed(mod, a, b, tz)
        exchange.complete(dev)
        for pair, (z, _), gate in zip(pairs, rz, gates):
            stages.trimul_output(mod, z, gate, pair)
        return
    projected = [stages.trimul_project(mod, pair, pair_mask[shard_rows(n, g, r)])
                 for pair, r in zip(pairs, exchange.ranks)]
    a_full, b_full = exchange.rows_to_channels_pair([a for a, _, _ in projected],
                                                    [b for _, b, _ in projected])  # [c/G, n, n]
    z = [stages.trimul_contract(mod, a, b) for a, b in zip(a_full, b_full)]
    del a_full, b_full
    z_rows = exchange.channels_to_rows(z)  # [c, rows, n]
    for pair, zr, (_, _, gate) in zip(pairs, z_rows, projected):
        stages.trimul_output(mod, zr, gate, pair)


def _attention(mod, pairs, pair_mask, exchange, stages):
    g = exchange.world
    rows, n, c = pairs[0].shape
    if not mod.transpose:
        prepared = [stages.attention_prepare(mod, pair) for pair in pairs]
        biases = exchange.gather_rows([bias for _, bias in prepared])
        for pair, (x, _), bias, r in zip(pairs, prepared, biases, exchange.ranks):
            stages.attention_rows(mod, x, pair_mask[shard_rows(n, g, r)], bias, out=pair)
        return
    # ending node: attention runs over pair columns; mask rows indexed by the column
    if _routed(exchange, stages):
        dev = pairs[0].device
        # the LayerNorm'd rows go to the column owners from the prepare kernel;
        # the bias gather's barrier publishes them too
        rx = exchange.route("transpose", (rows, n, c), torch.bfloat16, dev)
        bias_rows = [stages.attention_prepare_routed(mod, pair, tx)
                     for pair, (_, tx) in zip(pairs, rx)]
        biases = exchange.gather_rows(bias_rows)
        ru = exchange.route("transpose", (rows, n, c), torch.bfloat16, dev)
        for (xt, _), bias, r, (_, tu) in zip(rx, biases, exchange.ranks, ru):
            stages.attention_rows_routed(mod, xt, pair_mask[shard_rows(n, g, r)], bias, tu)
        exchange.complete(dev)
        for pair, (upd, _) in zip(pairs, ru):
            pair += upd
        return
    prepared = [stages.attention_prepare(mod, pair) for pair in pairs]
    biases = exchange.gather_rows([bias for _, bias in prepared])
    cols = exchange.transpose([x for x, _ in prepared])
    del prepared
    updates = [stages.attention_rows(mod, xt, pair_mask[shard_rows(n, g, r)], bias)
               for xt, bias, r in zip(cols, biases, exchange.ranks)]
    for pair, upd in zip(pairs, exchange.transpose(updates)):
        pair += upd


def pairformer_block(block: PairformerBlock, pairs: list[torch.Tensor], pair_mask: torch.Tensor,
                     single: torch.Tensor | None, seq_mask: torch.Tensor | None,
                     exchange, stages=None, single_stream=None, single_exchange=None):
    """One Pairformer block on a row-sharded pair, updated in place.

    pairs: this process's row blocks ([N/G, N, c] f32 contiguous, one per local
    shard, in `exchange.ranks` order); pair_mask: the full [N, N] mask (every
    process holds it); single / seq_mask: this process's copy of the single
    track, updated in place (once per process).

    The pair track never reads the single track, so with `single_stream` (a
    CUDA stream) and `single_exchange` (a second exchange of the same ranks,
    with its own buffers and barrier) the single track runs on that stream
    after the pair-logit rows and overlaps the next block's pair operators; the
    caller makes its stream wait for `single_stream` before reading `single`."""
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
    # single track sharded by query rows: each rank's pair-logit rows are the
    # bias rows of its own queries, so only the updated single rows are gathered
    logits = [stages.pair_logits_rows(block, pair) for pair in pairs]
    if single_stream is None:
        _single_track(block, single, seq_mask, logits, rows, exchange, stages)
        return pairs, single
    main = torch.cuda.current_stream(single.device)
    single_stream.wait_stream(main)
    for lg in logits:  # read on the side stream after the main stream drops them
        lg.record_stream(single_stream)
    with torch.cuda.stream(single_stream):
        _single_track(block, single, seq_mask, logits, rows, single_exchange, stages)
    return pairs, single


def _single_track(block, single, seq_mask, logits, rows, exchange, stages):
    x_in = single.clone() if len(logits) > 1 else single  # every shard reads the old single
    for lg, r in zip(logits, exchange.ranks):
        stages.single_attention_rows(block, x_in, seq_mask, lg, r * rows, single)
    for r in exchange.ranks:
        stages.single_transition_rows(block, single[r * rows:(r + 1) * rows])
    gathered = exchange.gather_rows([single[r * rows:(r + 1) * rows].unsqueeze(0)
                                     for r in exchange.ranks])
    single.copy_(gathered[0][0])
