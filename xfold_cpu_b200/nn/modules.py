"""xfold hot-path modules with the `cuda` backend.

Each class mirrors the reference module of the same name: constructor
arguments, submodule and parameter names (so a reference state_dict / AF3
checkpoint mapping loads unchanged) and forward signature.  forward() returns
the update like the reference; accumulate_() adds it into an f32 residual
stream in place through the fused epilogue (the `x += op(x)` of the callers).

  TriangleMultiplication   xfold/nn/triangle_multiplication.py:21-105
  GridSelfAttention        xfold/nn/attention.py:26-105
  Transition               xfold/nn/primitives.py:20-37
  AdaptiveLayerNorm        xfold/nn/diffusion_transformer.py:27-64
  AdaLNZero                xfold/nn/diffusion_transformer.py:67-95
  DiffusionTransition      xfold/nn/diffusion_transformer.py:98-128
  SelfAttention            xfold/nn/diffusion_transformer.py:131-217
  DiffusionTransformer     xfold/nn/diffusion_transformer.py:220-272
  MSAAttention             xfold/nn/attention.py:108-144
  OuterProductMean         xfold/nn/primitives.py:40-75
  EvoformerBlock           xfold/nn/pairformer.py:117-156
  CrossAttention           xfold/nn/diffusion_transformer.py:275-350
  DiffusionCrossAttTransformer  xfold/nn/diffusion_transformer.py:353-411
  PairformerBlock          xfold/nn/pairformer.py:26-114
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import fp32, native
from . import atom_layout
from ..fastnn import LayerNorm, WeightCache
from ..fastnn import config


def _bf16(cache: WeightCache, weight: torch.Tensor) -> torch.Tensor:
    return cache.get((weight,), native.prepare_weight)


def _f32_result(update: torch.Tensor, out, accumulate):
    """Hands an fp32-path update back the way the bf16 entry points do."""
    if out is None:
        return update
    if accumulate:
        out += update
    else:
        out.copy_(update)
    return out


def _fused_target(x: torch.Tensor) -> bool:
    """True when the update can be added in place by the kernel epilogue."""
    return x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()


class TriangleMultiplication(nn.Module):
    def __init__(self, c_pair: int = 128, _outgoing: bool = True) -> None:
        super().__init__()
        self.c_pair = c_pair
        self.left_norm_input = LayerNorm(c_pair)
        self.projection = nn.Linear(c_pair, 2 * c_pair, bias=False)
        self.gate = nn.Linear(c_pair, 2 * c_pair, bias=False)
        self.center_norm = LayerNorm(c_pair)
        self.output_projection = nn.Linear(c_pair, c_pair, bias=False)
        self.gating_linear = nn.Linear(c_pair, c_pair, bias=False)
        self.equation = "cik,cjk->cij" if _outgoing else "ckj,cki->cij"
        self._packed = WeightCache()
        self._out_w = WeightCache()

    @property
    def outgoing(self) -> bool:
        return self.equation == "cik,cjk->cij"

    def _run(self, pair, mask, out, accumulate):
        config.require_cuda("triangle_multiplication_implementation")
        if config.float32():
            return _f32_result(fp32.triangle_multiplication(self, pair, mask), out, accumulate)
        packed = self._packed.get(
            (self.projection.weight, self.gate.weight, self.gating_linear.weight),
            native.pack_triangle_weights)
        return native.triangle_multiplication(
            pair, mask, self.outgoing, self.left_norm_input.weight, self.left_norm_input.bias,
            None, None, self.center_norm.weight, self.center_norm.bias,
            _bf16(self._out_w, self.output_projection.weight), None,
            self.left_norm_input.eps, self.center_norm.eps, weights_packed=True, packed=packed,
            out=out, accumulate=accumulate)

    def forward(self, pair: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        return self._run(pair, mask, None, False)

    def accumulate_(self, pair: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        if _fused_target(pair):
            return self._run(pair, mask, pair, True)
        pair += self.forward(pair, mask)
        return pair


class GridSelfAttention(nn.Module):
    def __init__(self, c_pair: int = 128, num_head: int = 4, transpose: bool = False):
        super().__init__()
        self.c_pair = c_pair
        self.num_head = num_head
        self.qkv_dim = c_pair // num_head
        self.transpose = transpose
        self.act_norm = LayerNorm(c_pair)
        self.pair_bias_projection = nn.Linear(c_pair, num_head, bias=False)
        self.q_projection = nn.Linear(c_pair, c_pair, bias=False)
        self.k_projection = nn.Linear(c_pair, c_pair, bias=False)
        self.v_projection = nn.Linear(c_pair, c_pair, bias=False)
        self.gating_query = nn.Linear(c_pair, c_pair, bias=False)
        self.output_projection = nn.Linear(c_pair, c_pair, bias=False)
        self._packed = WeightCache()
        self._bias_w = WeightCache()
        self._out_w = WeightCache()

    def _run(self, pair, mask, out, accumulate):
        config.require_cuda("dot_product_attention_implementation")
        if config.float32():
            return _f32_result(fp32.grid_self_attention(self, pair, mask), out, accumulate)
        packed = self._packed.get(
            (self.q_projection.weight, self.k_projection.weight, self.v_projection.weight,
             self.gating_query.weight), native.pack_attention_weights)
        return native.grid_self_attention(
            pair, mask, self.transpose, self.act_norm.weight, self.act_norm.bias,
            self.act_norm.eps, _bf16(self._bias_w, self.pair_bias_projection.weight), packed,
            _bf16(self._out_w, self.output_projection.weight), self.num_head, out=out,
            accumulate=accumulate)

    def forward(self, pair: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        return self._run(pair, mask, None, False)

    def accumulate_(self, pair: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        if _fused_target(pair):
            return self._run(pair, mask, pair, True)
        pair += self.forward(pair, mask)
        return pair


class Transition(nn.Module):
    def __init__(self, c_x: int, num_intermediate_factor: int = 4) -> None:
        super().__init__()
        self.num_intermediate_factor = num_intermediate_factor
        self.c_in = c_x
        self.input_layer_norm = LayerNorm(c_x)
        self.transition1 = nn.Linear(c_x, num_intermediate_factor * c_x * 2, bias=False)
        self.transition2 = nn.Linear(num_intermediate_factor * c_x, c_x, bias=False)
        self._glu_weight_cache = WeightCache()
        self._w2 = WeightCache()

    def _run(self, x, out, accumulate):
        config.require_cuda("gated_linear_unit_implementation")
        if config.float32():
            return _f32_result(fp32.transition(self, x), out, accumulate)
        w1 = self._glu_weight_cache.get((self.transition1.weight,), native.pack_glu_weight)
        return native.transition(x, self.input_layer_norm.weight, self.input_layer_norm.bias,
                                 self.input_layer_norm.eps, w1,
                                 _bf16(self._w2, self.transition2.weight),
                                 self.num_intermediate_factor, out=out, accumulate=accumulate)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._run(x, None, False)

    def accumulate_(self, x: torch.Tensor) -> torch.Tensor:
        if _fused_target(x):
            return self._run(x, x, True)
        x += self.forward(x)
        return x


class AdaptiveLayerNorm(nn.Module):
    def __init__(self, c_x: int, c_single_cond: int, use_single_cond: bool = False) -> None:
        super().__init__()
        self.c_x = c_x
        self.c_single_cond = c_single_cond
        self.use_single_cond = use_single_cond
        if use_single_cond:
            self.layer_norm = LayerNorm(c_x, elementwise_affine=False, bias=False)
            self.single_cond_layer_norm = LayerNorm(c_single_cond, bias=False)
            self.single_cond_scale = nn.Linear(c_single_cond, c_x, bias=True)
            self.single_cond_bias = nn.Linear(c_single_cond, c_x, bias=False)
            self._cond_w = WeightCache()
        else:
            self.layer_norm = LayerNorm(c_x)

    def modulation(self, single_cond: torch.Tensor):
        """(sigmoid(scale), shift) of the conditioned path as bf16 [N, c_x]
        (:57-62): the library's LayerNorm and one conditioning GEMM against the
        stacked scale / shift weights, as DiffusionTransformer does for all of
        its blocks at once.  c_x must be a multiple of 64."""
        mod = _modulations(self._cond_w, [self], single_cond.reshape(-1, self.c_single_cond),
                           self.c_x)
        return mod[0], mod[1]

    def forward(self, x: torch.Tensor, single_cond: Optional[torch.Tensor] = None) -> torch.Tensor:
        assert (single_cond is None) == (self.use_single_cond is False)
        y = self.layer_norm(x)
        if self.use_single_cond:
            scale, shift = self.modulation(single_cond)
            return (scale.float() * y.float() + shift.float()).bfloat16()
        return y


class AdaLNZero(nn.Module):
    def __init__(self, c_in: int, c_out: int, c_single_cond: int, use_single_cond: bool = False) -> None:
        super().__init__()
        self.c_in = c_in
        self.c_out = c_out
        self.c_single_cond = c_single_cond
        self.use_single_cond = use_single_cond
        self.transition2 = nn.Linear(c_in, c_out, bias=False)
        if use_single_cond:
            self.adaptive_zero_cond = nn.Linear(c_single_cond, c_out, bias=True)
            self._gate_w = WeightCache()

    def out_gate(self, single_cond: torch.Tensor) -> torch.Tensor:
        """sigmoid(adaptive_zero_cond(single_cond)) as bf16 [N, c_out] (:91-94),
        one conditioning GEMM of the library.  c_out must be a multiple of 64."""
        return _gates(self._gate_w, [self], single_cond.reshape(-1, self.c_single_cond),
                      self.c_out)[0]

    def forward(self, x: torch.Tensor, single_cond: Optional[torch.Tensor] = None) -> torch.Tensor:
        assert (single_cond is None) == (self.use_single_cond is False)
        out = native.linear(x, self.transition2.weight)
        if self.use_single_cond:
            out = (self.out_gate(single_cond) * out).bfloat16()
        return out


class DiffusionTransition(nn.Module):
    def __init__(self, c_x: int, c_single_cond: int, num_intermediate_factor: int = 2,
                 use_single_cond: bool = False) -> None:
        super().__init__()
        self.c_x = c_x
        self.c_single_cond = c_single_cond
        self.num_intermediate_factor = num_intermediate_factor
        self.use_single_cond = use_single_cond
        self.adaptive_layernorm = AdaptiveLayerNorm(c_x, c_single_cond, use_single_cond)
        self.transition1 = nn.Linear(c_x, 2 * c_x * num_intermediate_factor, bias=False)
        self._glu_weight_cache = WeightCache()
        self.adaptive_zero_init = AdaLNZero(num_intermediate_factor * c_x, c_x, c_single_cond,
                                            use_single_cond)
        self._w2 = WeightCache()

    def _run(self, x, single_cond, out, accumulate, cond=None):
        config.require_cuda("gated_linear_unit_implementation")
        assert (single_cond is None) == (self.use_single_cond is False)
        if config.float32():
            return _f32_result(fp32.diffusion_transition(self, x, single_cond), out, accumulate)
        w1 = self._glu_weight_cache.get((self.transition1.weight,), native.pack_glu_weight)
        ln = self.adaptive_layernorm.layer_norm
        scale = shift = gate = None
        if cond is not None:  # (sigmoid(scale), shift, gate) computed for every block at once
            scale, shift, gate = cond
        elif self.use_single_cond:
            scale, shift = self.adaptive_layernorm.modulation(single_cond)
            gate = self.adaptive_zero_init.out_gate(single_cond)
        return native.transition(x, ln.weight, ln.bias, ln.eps, w1,
                                 _bf16(self._w2, self.adaptive_zero_init.transition2.weight),
                                 self.num_intermediate_factor, mod_scale=scale, mod_shift=shift,
                                 out_gate=gate, out=out, accumulate=accumulate)

    def forward(self, x: torch.Tensor, single_cond: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self._run(x, single_cond, None, False)

    def accumulate_(self, x, single_cond=None, cond=None):
        if _fused_target(x):
            return self._run(x, single_cond, x, True, cond)
        x += self._run(x, single_cond, None, False, cond)
        return x


class SelfAttention(nn.Module):
    def __init__(self, c_x: int = 768, c_single_cond: int = 384, num_head: int = 16,
                 use_single_cond: bool = False) -> None:
        super().__init__()
        self.c_x = c_x
        self.c_single_cond = c_single_cond
        self.num_head = num_head
        self.qkv_dim = c_x // num_head
        self.use_single_cond = use_single_cond
        self.adaptive_layernorm = AdaptiveLayerNorm(c_x, c_single_cond, use_single_cond)
        self.q_projection = nn.Linear(c_x, c_x, bias=True)
        self.k_projection = nn.Linear(c_x, c_x, bias=False)
        self.v_projection = nn.Linear(c_x, c_x, bias=False)
        self.gating_query = nn.Linear(c_x, c_x, bias=False)
        self.adaptive_zero_init = AdaLNZero(c_x, c_x, c_single_cond, use_single_cond)
        self._packed = WeightCache()
        self._wo = WeightCache()

    def _run(self, x, mask, pair_logits, single_cond, out, accumulate, cond=None):
        config.require_cuda("dot_product_attention_implementation")
        assert (single_cond is None) == (self.use_single_cond is False)
        if config.float32():
            return _f32_result(fp32.self_attention(self, x, mask, pair_logits, single_cond), out,
                               accumulate)
        packed = self._packed.get(
            (self.q_projection.weight, self.k_projection.weight, self.v_projection.weight,
             self.gating_query.weight), native.pack_attention_weights)
        ln = self.adaptive_layernorm.layer_norm
        scale = shift = gate = None
        if cond is not None:  # (sigmoid(scale), shift, gate) computed for every block at once
            scale, shift, gate = cond
        elif self.use_single_cond:
            scale, shift = self.adaptive_layernorm.modulation(single_cond)
            gate = self.adaptive_zero_init.out_gate(single_cond)
        return native.self_attention(
            x, mask, pair_logits, ln.weight, ln.bias, ln.eps, packed, self.q_projection.bias,
            _bf16(self._wo, self.adaptive_zero_init.transition2.weight), self.num_head,
            mod_scale=scale, mod_shift=shift, out_gate=gate, out=out, accumulate=accumulate)

    def forward(self, x: torch.Tensor, mask: torch.Tensor, pair_logits: Optional[torch.Tensor] = None,
                single_cond: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self._run(x, mask, pair_logits, single_cond, None, False)

    def accumulate_(self, x, mask, pair_logits=None, single_cond=None, cond=None):
        if _fused_target(x):
            return self._run(x, mask, pair_logits, single_cond, x, True, cond)
        x += self._run(x, mask, pair_logits, single_cond, None, False, cond)
        return x


def _modulations(cache: WeightCache, ada: list, single_cond: torch.Tensor, c: int) -> torch.Tensor:
    """(sigmoid(scale), shift) of every AdaptiveLayerNorm in `ada` from the same
    single_cond: [2 * len(ada), N, c] bf16, chunks (scale_0, shift_0, scale_1, ...).

    LayerNorm(single_cond) without its weight, then one GEMM against the
    modules' scale / shift weights with that LayerNorm weight folded in
    (diffusion_transformer.py:51-62 per module).  The modules share eps."""

    def build(*_):
        ws, bs = [], []
        for m in ada:
            g = m.single_cond_layer_norm.weight.float()
            ws += [m.single_cond_scale.weight.float() * g, m.single_cond_bias.weight.float() * g]
            bs += [m.single_cond_scale.bias.float(), torch.zeros_like(m.single_cond_scale.bias.float())]
        return torch.cat(ws).bfloat16().contiguous(), torch.cat(bs).contiguous()

    src = [t for m in ada for t in (m.single_cond_layer_norm.weight, m.single_cond_scale.weight,
                                    m.single_cond_scale.bias, m.single_cond_bias.weight)]
    w, b = cache.get(src, build)
    sc = native.layer_norm(single_cond, None, None, ada[0].single_cond_layer_norm.eps)
    return native.conditioning(sc, w, b, c, 1)


def _gates(cache: WeightCache, zero: list, single_cond: torch.Tensor, c: int) -> torch.Tensor:
    """sigmoid(adaptive_zero_cond(single_cond)) of every AdaLNZero in `zero`
    (diffusion_transformer.py:85-94): [len(zero), N, c] bf16, one GEMM."""

    def build(*_):
        w = torch.cat([z.adaptive_zero_cond.weight.float() for z in zero]).bfloat16()
        b = torch.cat([z.adaptive_zero_cond.bias.float() for z in zero])
        return w.contiguous(), b.contiguous()

    src = [t for z in zero for t in (z.adaptive_zero_cond.weight, z.adaptive_zero_cond.bias)]
    w, b = cache.get(src, build)
    return native.conditioning(single_cond, w, b, c, 2)


class DiffusionTransformer(nn.Module):
    def __init__(self, c_act: int = 768, c_single_cond: int = 384, c_pair_cond: int = 128,
                 num_head: int = 16, num_blocks: int = 24, super_block_size: int = 4) -> None:
        super().__init__()
        self.c_act = c_act
        self.c_single_cond = c_single_cond
        self.c_pair_cond = c_pair_cond
        self.num_head = num_head
        self.num_blocks = num_blocks
        self.super_block_size = super_block_size
        self.num_super_blocks = num_blocks // super_block_size
        self.pair_input_layer_norm = LayerNorm(c_pair_cond)
        self.pair_logits_projection = nn.ModuleList(
            [nn.Linear(c_pair_cond, super_block_size * num_head, bias=False)
             for _ in range(self.num_super_blocks)])
        self.self_attention = nn.ModuleList(
            [SelfAttention(c_act, c_single_cond, num_head=num_head, use_single_cond=True)
             for _ in range(num_blocks)])
        self.transition_block = nn.ModuleList(
            [DiffusionTransition(c_act, c_single_cond, use_single_cond=True)
             for _ in range(num_blocks)])
        self._logits_key = None
        self._logits = None
        self._cond_w = WeightCache()
        self._gate_w = WeightCache()

    def _adaln_modules(self):
        for i in range(self.num_blocks):
            yield self.self_attention[i].adaptive_layernorm
            yield self.transition_block[i].adaptive_layernorm

    def _zero_modules(self):
        for i in range(self.num_blocks):
            yield self.self_attention[i].adaptive_zero_init
            yield self.transition_block[i].adaptive_zero_init

    def conditioning(self, single_cond: torch.Tensor):
        """Every block's AdaLN (sigmoid(scale), shift) and AdaLNZero gate for one
        denoising step: the reference recomputes them in each block
        (diffusion_transformer.py:51-62, :85-94) from the same single_cond.

        LayerNorm(single_cond) without its weight, then one GEMM against the
        blocks' scale / shift weights with that LayerNorm weight folded in, and
        one GEMM of single_cond against the gate weights.  Returns per block
        (attention, transition) triples of contiguous [N, c_act] bf16 views."""
        ada = list(self._adaln_modules())
        zero = list(self._zero_modules())
        mod = _modulations(self._cond_w, ada, single_cond, self.c_act)  # [4 * blocks, N, c]
        gate = _gates(self._gate_w, zero, single_cond, self.c_act)  # [2 * blocks, N, c]
        return [((mod[4 * i], mod[4 * i + 1], gate[2 * i]),
                 (mod[4 * i + 2], mod[4 * i + 3], gate[2 * i + 1])) for i in range(self.num_blocks)]

    def pair_logits(self, pair_cond: torch.Tensor) -> list[torch.Tensor]:
        """[super_block][j] -> [H, N, N] bf16 logits; cached per pair_cond version
        like the reference's InputCache (:256-265)."""
        try:
            key = (pair_cond.data_ptr(), pair_cond._version, tuple(pair_cond.shape),
                   tuple((p.weight.data_ptr(), p.weight._version)
                         for p in self.pair_logits_projection))
        except RuntimeError:  # inference tensors carry no version counter: no reuse
            key = None
        if key is not None:
            key = (key, config.compute_dtype)
        if key is None or key != self._logits_key:
            ln = self.pair_input_layer_norm
            logits = []
            if config.float32():
                n = pair_cond.shape[0]
                x = fp32.layer_norm(pair_cond, ln.weight, ln.bias, ln.eps)
                for proj in self.pair_logits_projection:
                    w = proj.weight.float()  # [(b h), c]: block j uses rows [j*H, (j+1)*H)
                    out = torch.empty((w.shape[0], n, n), dtype=torch.float32, device=x.device)
                    fp32.gemm(x.view(1, n * n, -1), w.unsqueeze(0),
                              out.view(w.shape[0], n * n).t().unsqueeze(0))
                    logits.append([out[j * self.num_head:(j + 1) * self.num_head]
                                   for j in range(self.super_block_size)])
            else:
                for proj in self.pair_logits_projection:
                    w = proj.weight  # [(b h), c]: block j uses rows [j*H, (j+1)*H)
                    logits.append([native.pair_logits(pair_cond, ln.weight, ln.bias, ln.eps,
                                                      w[j * self.num_head:(j + 1) * self.num_head])
                                   for j in range(self.super_block_size)])
            self._logits, self._logits_key = logits, key
        return self._logits

    def run_blocks(self, act: torch.Tensor, mask: torch.Tensor, single_cond: torch.Tensor,
                   logits: list[list[torch.Tensor]]) -> torch.Tensor:
        """The blocks of forward() with the pair logits given (act updated in place);
        the conditioning of all blocks is computed first, in one pass."""
        # the fp32 path conditions each block from single_cond itself
        cond = None if config.float32() else self.conditioning(single_cond)
        for s in range(self.num_super_blocks):
            for j in range(self.super_block_size):
                i = s * self.super_block_size + j
                self.self_attention[i].accumulate_(act, mask, logits[s][j], single_cond,
                                                   cond=None if cond is None else cond[i][0])
                self.transition_block[i].accumulate_(act, single_cond,
                                                     cond=None if cond is None else cond[i][1])
        return act

    def forward(self, act: torch.Tensor, mask: torch.Tensor, single_cond: torch.Tensor,
                pair_cond: torch.Tensor) -> torch.Tensor:
        return self.run_blocks(act, mask, single_cond, self.pair_logits(pair_cond))

    def capture(self, act: torch.Tensor, mask: torch.Tensor, single_cond: torch.Tensor,
                pair_cond: torch.Tensor) -> "DiffusionStepGraph":
        """Records the transformer's blocks for these shapes into a CUDA graph.

        The reference runs this transformer 24 blocks deep at every denoising
        step of every sample (xfold/alphafold3.py:328-395 call the diffusion
        head, xfold/nn/diffusion_head.py:234 calls the transformer) with the
        pair conditioning fixed: its logits are computed here once,
        and each replay launches every kernel of the 24 blocks with one call.
        The tensors given are copied into the graph's own input buffers; see
        DiffusionStepGraph for replaying with new act / single_cond."""
        return DiffusionStepGraph(self, act, mask, single_cond, pair_cond)


class DiffusionStepGraph:
    """A CUDA graph of DiffusionTransformer.run_blocks for fixed shapes and
    pair conditioning.  __call__(act, single_cond) copies the inputs into the
    graph's buffers, replays the graph on the current stream and returns the
    graph's output buffer (overwritten by the next call)."""

    def __init__(self, module: DiffusionTransformer, act, mask, single_cond, pair_cond) -> None:
        self.module = module
        self.logits = module.pair_logits(pair_cond)
        self.act = act.detach().clone()
        self.mask = mask.detach().clone()
        self.single_cond = single_cond.detach().clone()
        work = self.act.clone()
        # warm-up on a side stream: weight caches filled, kernels' attributes set
        side = torch.cuda.Stream(device=self.act.device)
        side.wait_stream(torch.cuda.current_stream(self.act.device))
        with torch.cuda.stream(side):
            module.run_blocks(work, self.mask, self.single_cond, self.logits)
        torch.cuda.current_stream(self.act.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self.act.clone()
            module.run_blocks(self.out, self.mask, self.single_cond, self.logits)

    def __call__(self, act: torch.Tensor, single_cond: torch.Tensor) -> torch.Tensor:
        self.act.copy_(act)
        self.single_cond.copy_(single_cond)
        self.graph.replay()
        return self.out


class CrossAttention(nn.Module):
    """Windowed cross-attention of the atom transformer: 32 queries x 128 keys
    per subset, c = 128, 4 heads (the sizes DiffusionCrossAttTransformer builds);
    other sizes raise ValueError."""

    def __init__(self, key_dim: int = 128, value_dim: int = 128, c_single_cond: int = 128,
                 num_head: int = 4) -> None:
        super().__init__()
        self.key_dim = key_dim
        self.value_dim = value_dim
        self.c_single_cond = c_single_cond
        self.num_head = num_head
        self.key_dim_per_head = key_dim // num_head
        self.value_dim_per_head = value_dim // num_head
        self.q_scale = self.key_dim_per_head ** (-0.5)
        self.q_adaptive_layernorm = AdaptiveLayerNorm(key_dim, c_single_cond, use_single_cond=True)
        self.k_adaptive_layernorm = AdaptiveLayerNorm(key_dim, c_single_cond, use_single_cond=True)
        self.q_projection = nn.Linear(key_dim, key_dim, bias=True)
        self.k_projection = nn.Linear(key_dim, key_dim, bias=False)
        self.v_projection = nn.Linear(value_dim, value_dim, bias=False)
        self.gating_query = nn.Linear(key_dim, value_dim, bias=False)
        self.adaptive_zero_init = AdaLNZero(value_dim, value_dim, key_dim, use_single_cond=True)
        self._packed = WeightCache()
        self._wo = WeightCache()

    def _run(self, x_q, keys, mask_q, mask_k, pair_logits, single_cond_q, single_cond_k, out,
             accumulate, cond=None):
        config.require_cuda("dot_product_attention_implementation")
        if (self.key_dim, self.value_dim, self.num_head) != (128, 128, 4):
            raise ValueError("the cuda backend's cross-attention takes key_dim = value_dim = 128, "
                             "4 heads")
        packed = self._packed.get(
            (self.q_projection.weight, self.gating_query.weight, self.k_projection.weight,
             self.v_projection.weight), native.pack_cross_attention_weights)
        if cond is not None:  # (q_scale, q_shift, k_scale, k_shift, gate), all blocks at once
            qs, qh, ks, kh, gate = cond
        else:
            qs, qh = self.q_adaptive_layernorm.modulation(single_cond_q.reshape(-1, self.c_single_cond))
            ks, kh = self.k_adaptive_layernorm.modulation(single_cond_k.reshape(-1, self.c_single_cond))
            gate = self.adaptive_zero_init.out_gate(single_cond_q.reshape(-1, self.c_single_cond))
        eps = self.q_adaptive_layernorm.layer_norm.eps
        return native.cross_attention(
            x_q, keys, mask_q, mask_k, pair_logits, eps, packed, self.q_projection.bias,
            _bf16(self._wo, self.adaptive_zero_init.transition2.weight), q_mod=(qs, qh),
            k_mod=(ks, kh), out_gate=gate, out=out, accumulate=accumulate)

    def forward(self, x_q: torch.Tensor, x_k: torch.Tensor, mask_q: torch.Tensor,
                mask_k: torch.Tensor, pair_logits: Optional[torch.Tensor] = None,
                single_cond_q: Optional[torch.Tensor] = None,
                single_cond_k: Optional[torch.Tensor] = None) -> torch.Tensor:
        assert mask_q.dim() == x_q.dim() - 1 and mask_k.dim() == x_k.dim() - 1
        return self._run(x_q, x_k, mask_q, mask_k, pair_logits, single_cond_q, single_cond_k,
                         None, False)

    def accumulate_(self, x_q, keys, mask_q, mask_k, pair_logits=None, single_cond_q=None,
                    single_cond_k=None, cond=None):
        """x_q += forward(...), with keys either x_k or the (index, valid) gather
        of x_q's rows (atom_layout.key_gather)."""
        if _fused_target(x_q):
            return self._run(x_q, keys, mask_q, mask_k, pair_logits, single_cond_q, single_cond_k,
                             x_q, True, cond)
        x_q += self._run(x_q, keys, mask_q, mask_k, pair_logits, single_cond_q, single_cond_k,
                         None, False, cond)
        return x_q


class DiffusionCrossAttTransformer(nn.Module):
    def __init__(self, c_query: int = 128, c_single_cond: int = 128, c_pair_cond: int = 16,
                 num_blocks: int = 3, num_head: int = 4) -> None:
        super().__init__()
        self.c_query = c_query
        self.c_single_cond = c_single_cond
        self.c_pair_cond = c_pair_cond
        self.num_blocks = num_blocks
        self.num_head = num_head
        self.pair_input_layer_norm = LayerNorm(c_pair_cond, bias=False)
        self.pair_logits_projection = nn.Linear(c_pair_cond, num_blocks * num_head, bias=False)
        self.cross_attention = nn.ModuleList(
            [CrossAttention(num_head=num_head) for _ in range(num_blocks)])
        self.transition_block = nn.ModuleList(
            [DiffusionTransition(c_x=c_query, c_single_cond=c_single_cond, use_single_cond=True)
             for _ in range(num_blocks)])
        self._logits_key = None
        self._logits = None
        self._gather_key = None
        self._gather = None
        self._q_mod_w = WeightCache()
        self._k_mod_w = WeightCache()
        self._gate_w = WeightCache()

    def pair_logits(self, pair_cond: torch.Tensor) -> torch.Tensor:
        """[blocks, subsets, heads, q, k] bf16, cached per pair_cond version like
        the reference's InputCache (diffusion_transformer.py:376-380)."""
        try:
            key = (pair_cond.data_ptr(), pair_cond._version, tuple(pair_cond.shape),
                   self.pair_logits_projection.weight.data_ptr(),
                   self.pair_logits_projection.weight._version,
                   self.pair_input_layer_norm.weight.data_ptr(),
                   self.pair_input_layer_norm.weight._version)
        except RuntimeError:  # inference tensors carry no version counter: no reuse
            key = None
        if key is None or key != self._logits_key:
            ln = self.pair_input_layer_norm
            self._logits = native.cross_pair_logits(pair_cond, ln.weight, ln.bias, ln.eps,
                                                    self.pair_logits_projection.weight,
                                                    self.num_blocks, self.num_head)
            self._logits_key = key
        return self._logits

    def key_gather(self, queries_to_keys, source_rows: int, device: torch.device):
        """(index, valid) of the keys on the device, cached per GatherInfo."""
        try:
            key = (queries_to_keys.gather_idxs.data_ptr(), queries_to_keys.gather_idxs._version,
                   queries_to_keys.gather_mask.data_ptr(), queries_to_keys.gather_mask._version,
                   source_rows, device)
        except RuntimeError:
            key = None
        if key is None or key != self._gather_key:
            self._gather = atom_layout.key_gather(queries_to_keys, source_rows, device)
            self._gather_key = key
        return self._gather

    def conditioning(self, queries_single_cond: torch.Tensor, keys_single_cond: torch.Tensor):
        """Every block's conditioning for one call: per block
        ((q_scale, q_shift, k_scale, k_shift, attention gate),
         (transition scale, transition shift, transition gate)), [rows, c] bf16.
        The reference recomputes each from the same single conditionings."""
        c = self.c_query
        qsc = queries_single_cond.reshape(-1, self.c_single_cond)
        ksc = keys_single_cond.reshape(-1, self.c_single_cond)
        q_ada, zero, k_ada = [], [], []
        for i in range(self.num_blocks):
            q_ada += [self.cross_attention[i].q_adaptive_layernorm,
                      self.transition_block[i].adaptive_layernorm]
            zero += [self.cross_attention[i].adaptive_zero_init,
                     self.transition_block[i].adaptive_zero_init]
            k_ada.append(self.cross_attention[i].k_adaptive_layernorm)
        qm = _modulations(self._q_mod_w, q_ada, qsc, c)  # [4 * blocks, rows_q, c]
        km = _modulations(self._k_mod_w, k_ada, ksc, c)  # [2 * blocks, rows_k, c]
        gate = _gates(self._gate_w, zero, qsc, c)  # [2 * blocks, rows_q, c]
        return [((qm[4 * i], qm[4 * i + 1], km[2 * i], km[2 * i + 1], gate[2 * i]),
                 (qm[4 * i + 2], qm[4 * i + 3], gate[2 * i + 1])) for i in range(self.num_blocks)]

    def run_blocks(self, queries_act, queries_mask, keys, keys_mask, queries_single_cond,
                   keys_single_cond, logits):
        """The blocks of forward() with the pair logits and the key gather given."""
        cond = self.conditioning(queries_single_cond, keys_single_cond)
        # f32 masks once for all blocks (the kernels read 0 = masked)
        queries_mask = queries_mask.to(torch.float32).contiguous()
        keys_mask = keys_mask.to(torch.float32).contiguous()
        for i in range(self.num_blocks):
            self.cross_attention[i].accumulate_(queries_act, keys, queries_mask, keys_mask,
                                                logits[i], queries_single_cond, keys_single_cond,
                                                cond=cond[i][0])
            self.transition_block[i].accumulate_(queries_act, queries_single_cond, cond=cond[i][1])
        return queries_act

    def forward(self, queries_act: torch.Tensor, queries_mask: torch.Tensor, queries_to_keys,
                keys_mask: torch.Tensor, queries_single_cond: torch.Tensor,
                keys_single_cond: torch.Tensor, pair_cond: torch.Tensor) -> torch.Tensor:
        """Updates queries_act [subsets, queries, c] in place and returns it."""
        s, nq, _ = queries_act.shape
        keys = self.key_gather(queries_to_keys, s * nq, queries_act.device)
        return self.run_blocks(queries_act, queries_mask, keys, keys_mask, queries_single_cond,
                               keys_single_cond, self.pair_logits(pair_cond))

    def capture(self, queries_act, queries_mask, queries_to_keys, keys_mask, queries_single_cond,
                keys_single_cond, pair_cond) -> "CrossAttStepGraph":
        """Records the transformer's blocks for these shapes, masks, gather and
        pair conditioning into a CUDA graph (the encoder and the decoder call
        it at every denoising step, xfold/nn/atom_cross_attention.py:226-234,
        :408-416); see CrossAttStepGraph."""
        return CrossAttStepGraph(self, queries_act, queries_mask, queries_to_keys, keys_mask,
                                 queries_single_cond, keys_single_cond, pair_cond)


class CrossAttStepGraph:
    """A CUDA graph of DiffusionCrossAttTransformer.run_blocks.  __call__(act,
    queries_single_cond, keys_single_cond) copies the inputs into the graph's
    buffers, replays it on the current stream and returns the graph's output
    buffer (overwritten by the next call)."""

    def __init__(self, module: DiffusionCrossAttTransformer, act, queries_mask, queries_to_keys,
                 keys_mask, queries_single_cond, keys_single_cond, pair_cond) -> None:
        s, nq, _ = act.shape
        self.module = module
        self.logits = module.pair_logits(pair_cond)
        self.keys = tuple(t.clone() for t in module.key_gather(queries_to_keys, s * nq, act.device))
        self.act = act.detach().clone()
        self.qmask = queries_mask.detach().clone()
        self.kmask = keys_mask.detach().clone()
        self.qsc = queries_single_cond.detach().clone()
        self.ksc = keys_single_cond.detach().clone()
        args = (self.qmask, self.keys, self.kmask, self.qsc, self.ksc, self.logits)
        work = self.act.clone()
        side = torch.cuda.Stream(device=self.act.device)
        side.wait_stream(torch.cuda.current_stream(self.act.device))
        with torch.cuda.stream(side):
            module.run_blocks(work, *args)
        torch.cuda.current_stream(self.act.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self.act.clone()
            module.run_blocks(self.out, *args)

    def __call__(self, act: torch.Tensor, queries_single_cond: torch.Tensor,
                 keys_single_cond: torch.Tensor) -> torch.Tensor:
        self.act.copy_(act)
        self.qsc.copy_(queries_single_cond)
        self.ksc.copy_(keys_single_cond)
        self.graph.replay()
        return self.out


class MSAAttention(nn.Module):
    def __init__(self, c_msa: int = 64, c_pair: int = 128, num_head: int = 8) -> None:
        super().__init__()
        self.c_msa = c_msa
        self.c_pair = c_pair
        self.num_head = num_head
        self.value_dim = c_msa // num_head
        self.act_norm = LayerNorm(c_msa)
        self.pair_norm = LayerNorm(c_pair)
        self.pair_logits = nn.Linear(c_pair, num_head, bias=False)
        self.v_projection = nn.Linear(c_msa, num_head * self.value_dim, bias=False)
        self.gating_query = nn.Linear(c_msa, c_msa, bias=False)
        self.output_projection = nn.Linear(c_msa, c_msa, bias=False)
        self._w = [WeightCache() for _ in range(4)]

    def _run(self, msa, msa_mask, pair, out, accumulate):
        config.require_cuda("dot_product_attention_implementation")
        if (self.c_msa, self.c_pair, self.num_head) != (64, 128, 8):
            raise ValueError("the cuda backend's MSA attention takes c_msa = 64, c_pair = 128, "
                             "8 heads")
        w = [_bf16(c, t.weight) for c, t in zip(self._w, (self.pair_logits, self.v_projection,
                                                           self.gating_query,
                                                           self.output_projection))]
        return native.msa_attention(msa, msa_mask, pair, self.act_norm.weight, self.act_norm.bias,
                                    self.pair_norm.weight, self.pair_norm.bias, self.act_norm.eps,
                                    *w, out=out, accumulate=accumulate)

    def forward(self, msa: torch.Tensor, msa_mask: torch.Tensor, pair: torch.Tensor) -> torch.Tensor:
        return self._run(msa, msa_mask, pair, None, False)

    def accumulate_(self, msa, msa_mask, pair):
        if _fused_target(msa):
            return self._run(msa, msa_mask, pair, msa, True)
        msa += self._run(msa, msa_mask, pair, None, False)
        return msa


class OuterProductMean(nn.Module):
    def __init__(self, c_msa: int = 64, num_output_channel: int = 128,
                 num_outer_channel: int = 32) -> None:
        super().__init__()
        self.c_msa = c_msa
        self.num_outer_channel = num_outer_channel
        self.num_output_channel = num_output_channel
        self.epsilon = 1e-3
        self.layer_norm_input = LayerNorm(c_msa)
        self.left_projection = nn.Linear(c_msa, num_outer_channel, bias=False)
        self.right_projection = nn.Linear(c_msa, num_outer_channel, bias=False)
        self.output_w = nn.Parameter(torch.randn(num_outer_channel, num_outer_channel,
                                                 num_output_channel))
        self.output_b = nn.Parameter(torch.randn(num_output_channel))
        self._lw, self._rw, self._ow = WeightCache(), WeightCache(), WeightCache()

    def _run(self, msa, mask, out, accumulate):
        config.require_cuda("triangle_multiplication_implementation")
        if (self.c_msa, self.num_outer_channel, self.num_output_channel) != (64, 32, 128):
            raise ValueError("the cuda backend's outer product mean takes c_msa = 64, 32 outer "
                             "and 128 output channels")
        ln = self.layer_norm_input
        return native.outer_product_mean(
            msa, mask, ln.weight, ln.bias, ln.eps, _bf16(self._lw, self.left_projection.weight),
            _bf16(self._rw, self.right_projection.weight),
            self._ow.get((self.output_w,), native.pack_outer_product_weight), self.output_b,
            out=out, accumulate=accumulate)

    def forward(self, msa: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
        return self._run(msa, mask, None, False)

    def accumulate_(self, pair, msa, mask):
        """pair += forward(msa, mask), added by the kernel into an f32 pair."""
        if _fused_target(pair):
            return self._run(msa, mask, pair, True)
        pair += self._run(msa, mask, None, False)
        return pair


class EvoformerBlock(nn.Module):
    def __init__(self, c_msa: int = 64, c_pair: int = 128, n_heads_pair: int = 4) -> None:
        super().__init__()
        self.outer_product_mean = OuterProductMean(c_msa=c_msa, num_output_channel=c_pair)
        self.msa_attention1 = MSAAttention(c_msa=c_msa, c_pair=c_pair)
        self.msa_transition = Transition(c_x=c_msa)
        self.triangle_multiplication_outgoing = TriangleMultiplication(c_pair=c_pair, _outgoing=True)
        self.triangle_multiplication_incoming = TriangleMultiplication(c_pair=c_pair, _outgoing=False)
        self.pair_attention1 = GridSelfAttention(c_pair=c_pair, num_head=n_heads_pair, transpose=False)
        self.pair_attention2 = GridSelfAttention(c_pair=c_pair, num_head=n_heads_pair, transpose=True)
        self.pair_transition = Transition(c_x=c_pair)

    def forward(self, msa: torch.Tensor, pair: torch.Tensor, msa_mask: torch.Tensor,
                pair_mask: torch.Tensor):
        """Updates msa and pair in place and returns them, as the reference."""
        self.outer_product_mean.accumulate_(pair, msa, msa_mask)
        self.msa_attention1.accumulate_(msa, msa_mask, pair)
        self.msa_transition.accumulate_(msa)
        self.triangle_multiplication_outgoing.accumulate_(pair, pair_mask)
        self.triangle_multiplication_incoming.accumulate_(pair, pair_mask)
        self.pair_attention1.accumulate_(pair, pair_mask)
        self.pair_attention2.accumulate_(pair, pair_mask)
        self.pair_transition.accumulate_(pair)
        return msa, pair


class PairformerBlock(nn.Module):
    def __init__(self, n_heads: int = 16, c_pair: int = 128, c_single: int = 384,
                 c_hidden_mul: int = 128, n_heads_pair: int = 4, num_intermediate_factor: int = 4,
                 with_single: bool = True) -> None:
        super().__init__()
        self.n_heads = n_heads
        self.with_single = with_single
        self.num_intermediate_factor = num_intermediate_factor
        self.triangle_multiplication_outgoing = TriangleMultiplication(c_pair=c_pair, _outgoing=True)
        self.triangle_multiplication_incoming = TriangleMultiplication(c_pair=c_pair, _outgoing=False)
        self.pair_attention1 = GridSelfAttention(c_pair=c_pair, num_head=n_heads_pair, transpose=False)
        self.pair_attention2 = GridSelfAttention(c_pair=c_pair, num_head=n_heads_pair, transpose=True)
        self.pair_transition = Transition(c_x=c_pair, num_intermediate_factor=num_intermediate_factor)
        self.c_single = c_single
        if with_single:
            self.single_pair_logits_norm = LayerNorm(c_pair)
            self.single_pair_logits_projection = nn.Linear(c_pair, n_heads, bias=False)
            self.single_attention_ = SelfAttention(c_x=c_single, num_head=n_heads, use_single_cond=False)
            self.single_transition = Transition(c_x=c_single)
        self._logits_w = WeightCache()

    def forward(self, pair: torch.Tensor, pair_mask: torch.Tensor,
                single: Optional[torch.Tensor] = None, seq_mask: Optional[torch.Tensor] = None):
        """Updates pair (and single) in place and returns them, as the reference."""
        self.triangle_multiplication_outgoing.accumulate_(pair, pair_mask)
        self.triangle_multiplication_incoming.accumulate_(pair, pair_mask)
        self.pair_attention1.accumulate_(pair, pair_mask)
        self.pair_attention2.accumulate_(pair, pair_mask)
        self.pair_transition.accumulate_(pair)
        if not self.with_single:
            return pair
        norm = self.single_pair_logits_norm
        if config.float32():
            logits = fp32.pair_logits(self, pair)
        else:
            logits = native.pair_logits(pair, norm.weight, norm.bias, norm.eps,
                                        _bf16(self._logits_w,
                                              self.single_pair_logits_projection.weight))
        self.single_attention_.accumulate_(single, seq_mask, logits)
        self.single_transition.accumulate_(single)
        return pair, single
