"""Row-block stages of the reference algorithm, float32 on the CPU.

Test infrastructure (like the rest of oracle/): it lets the row-sharded
Pairformer driver (xfold_cpu_b200/sharded.py) run with gloo ranks on the CPU so
that its exchange steps can be checked against the whole-pair restatement in
oracle/hotpath.py.  Each method computes one stage of the reference operator on
a block of pair rows, with the tensor layouts of the library's row-block entry
points (a, b and z channel-major [c, rows, n]; bias [heads, rows, n]):

* TriangleMultiplication._forward_torch, xfold/nn/triangle_multiplication.py:71-105
  (projection :81-95, einsum :34-36, centre LN and output :96-105);
* GridSelfAttention.forward, xfold/nn/attention.py:80-105 (LN and bias :86-98,
  attention on rows :61-78 with the un-transposed mask :99-100);
* Transition, xfold/nn/primitives.py:33-37;
* the single track, xfold/nn/pairformer.py:102-112, by query rows.
"""

from __future__ import annotations

import torch

from .hotpath import (dot_product_attention, layer_norm, linear, self_attention, transition)


def _sd(module) -> dict:
    return {k: v.detach().float() for k, v in module.state_dict().items()}


class OracleStages:
    """Same interface as xfold_cpu_b200.sharded.NativeStages, in float32 torch."""

    def trimul_project(self, mod, pair_rows, mask_rows):
        rows, n, c = pair_rows.shape
        x = layer_norm(pair_rows, mod.left_norm_input.weight, mod.left_norm_input.bias)
        proj = linear(x, mod.projection.weight).permute(2, 0, 1)
        if mask_rows is not None:
            proj = proj * mask_rows[None]
        proj = proj * torch.sigmoid(linear(x, mod.gate.weight).permute(2, 0, 1))
        proj = proj.reshape(c, 2, rows, n)
        gate = torch.sigmoid(linear(x, mod.gating_linear.weight))
        return proj[:, 0].contiguous(), proj[:, 1].contiguous(), gate

    def trimul_contract(self, mod, a, b):
        equation = "cik,cjk->cij" if mod.outgoing else "ckj,cki->cij"
        return torch.einsum(equation, a, b)

    def trimul_output(self, mod, z_rows, g, pair_rows):
        z = layer_norm(z_rows.permute(1, 2, 0), mod.center_norm.weight, mod.center_norm.bias)
        pair_rows += linear(z, mod.output_projection.weight) * g

    def attention_prepare(self, mod, pair_rows):
        x = layer_norm(pair_rows, mod.act_norm.weight, mod.act_norm.bias)
        return x, linear(x, mod.pair_bias_projection.weight).permute(2, 0, 1).contiguous()

    def attention_rows(self, mod, x_rows, mask_rows, bias, out=None):
        rows, n, c = x_rows.shape
        h = mod.num_head
        d = c // h

        def heads(t):
            return t.reshape(rows, n, h, d).permute(0, 2, 1, 3)

        q = heads(linear(x_rows, mod.q_projection.weight))
        k = heads(linear(x_rows, mod.k_projection.weight))
        v = heads(linear(x_rows, mod.v_projection.weight))
        o = dot_product_attention(q, k, v, mask=mask_rows, bias=bias)
        o = o.permute(0, 2, 1, 3).reshape(rows, n, c)
        o = o * torch.sigmoid(linear(x_rows, mod.gating_query.weight))
        update = linear(o, mod.output_projection.weight)
        if out is None:
            return update
        out += update
        return out

    def transition(self, block, pair_rows):
        pair_rows += transition(pair_rows, _sd(block.pair_transition))

    def pair_logits_rows(self, block, pair_rows):
        norm = block.single_pair_logits_norm
        x = layer_norm(pair_rows, norm.weight, norm.bias)
        return linear(x, block.single_pair_logits_projection.weight).permute(2, 0, 1).contiguous()

    def single_attention_rows(self, block, x, seq_mask, logits_rows, row0, out):
        """The single attention update of query rows [row0, row0 + q_rows): the
        whole-track restatement with those rows' logits (queries are
        independent, so the other logit rows do not matter)."""
        heads, q_rows, n = logits_rows.shape
        logits = torch.zeros((heads, n, n), dtype=torch.float32)
        logits[:, row0:row0 + q_rows] = logits_rows.float()
        upd = self_attention(x, seq_mask, logits, _sd(block.single_attention_), None,
                             block.n_heads, False)
        out[row0:row0 + q_rows] += upd[row0:row0 + q_rows]

    def single_transition_rows(self, block, single_rows):
        single_rows += transition(single_rows, _sd(block.single_transition))
