"""CPU oracle of xfold's Pairformer / diffusion hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU in float32, the algorithm of
the reference implementation (Zhengye-AIsys/xfold_cpu, torch backend) for
every operator the CUDA library replaces.  Each function cites the reference
file:line it follows.  It is the checker for the parity tests, the smoke test
and bench.py's cpu_baseline / reference arm; the product path never imports
it (the CUDA library raises instead of falling back).

Parity pin: the restatement is checked against golden vectors produced by
running the reference modules themselves (tests/golden/make_golden.py, which
imports the reference checkout; fixtures in tests/golden/*.npz).

Parameters are dicts keyed by the reference modules' state_dict names, so a
module's state_dict (moved to the CPU) can be passed in directly.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _p(params: dict, prefix: str, name: str):
    return params.get(f"{prefix}{name}")


# --------------------------------------------------------------------------- primitives

def layer_norm(x, weight=None, bias=None, eps=1e-5):
    """fastnn.LayerNorm torch path: F.layer_norm over the last dim
    (xfold/fastnn/layer_norm.py:55-59), eps 1e-5 (:18)."""
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def linear(x, weight, bias=None):
    """nn.Linear: x @ W^T (+ b)."""
    y = x @ weight.T
    return y if bias is None else y + bias


def gated_linear_unit(x, weight_t):
    """gated_linear_unit_torch (xfold/fastnn/gated_linear_unit.py:103-107):
    y = x @ W; a, b = chunk(y, 2); silu(a) * b.  weight_t is [K, 2N]."""
    y = x @ weight_t
    a, b = torch.chunk(y, 2, dim=-1)
    return F.silu(a) * b


def dot_product_attention(q, k, v, mask=None, bias=None, query_chunk=None):
    """dot_product_attention_torch (xfold/fastnn/attention.py:45-66) with the 3-D
    unsqueeze of the dispatcher (:74-79, :95-96).

    q is scaled by d^-0.5 before QK^T; bias is added; masked logits are
    replaced by -1e9 (mask rank 1 -> [1,1,1,K], rank 2 -> [B,1,1,K], else a
    broadcastable bool); softmax over keys; weights @ v.  `query_chunk`
    processes batch rows in slices to bound memory (same arithmetic)."""
    squeeze = q.dim() == 3
    if squeeze:
        q, k, v = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0)
    if mask is not None:
        if mask.dim() == 1:
            mask = mask[None, None, None, :].to(dtype=torch.bool)
        elif mask.dim() == 2:
            mask = mask[:, None, None, :].to(dtype=torch.bool)
    B = q.shape[0]
    chunk = B if query_chunk is None else max(1, query_chunk)
    outs = []
    scaling = q.size(-1) ** -0.5
    for s in range(0, B, chunk):
        e = min(B, s + chunk)
        qq = q[s:e] * scaling
        logits = torch.matmul(qq, k[s:e].transpose(-1, -2))
        if bias is not None:
            bb = bias if bias.dim() < 4 or bias.shape[0] == 1 else bias[s:e]
            logits = logits + bb
        if mask is not None:
            mm = mask if mask.shape[0] == 1 else mask[s:e]
            logits = logits.masked_fill(~mm, -1e9)
        weights = torch.softmax(logits, dim=-1)
        outs.append(torch.matmul(weights, v[s:e]))
    out = torch.cat(outs, dim=0) if len(outs) > 1 else outs[0]
    return out.squeeze(0) if squeeze else out


# --------------------------------------------------------------------------- modules

def triangle_multiplication(pair, mask, params, outgoing, prefix=""):
    """TriangleMultiplication._forward_torch (xfold/nn/triangle_multiplication.py:71-105).

    x = LN(pair); proj = (x Wp^T) permuted to [2c, N, N] and multiplied by the
    mask; proj *= sigmoid(x Wg^T); a = proj[0::2], b = proj[1::2] (reshape to
    [c, 2, N, N], :92-95); einsum 'cik,cjk->cij' (outgoing) or 'ckj,cki->cij'
    (incoming) (:34-36); centre LN over c; output projection; times
    sigmoid(x W_gl^T).  Returns the update."""
    P = lambda n: _p(params, prefix, n)
    c = pair.shape[-1]
    x = layer_norm(pair, P("left_norm_input.weight"), P("left_norm_input.bias"))
    proj = linear(x, P("projection.weight")).permute(2, 0, 1)
    if mask is not None:
        proj = proj * mask[None, ...]
    gate = linear(x, P("gate.weight")).permute(2, 0, 1)
    proj = proj * torch.sigmoid(gate)
    proj = proj.reshape(c, 2, *proj.shape[1:])
    a, b = proj[:, 0], proj[:, 1]
    equation = "cik,cjk->cij" if outgoing else "ckj,cki->cij"
    z = torch.einsum(equation, a, b).permute(1, 2, 0)
    z = layer_norm(z, P("center_norm.weight"), P("center_norm.bias"))
    z = linear(z, P("output_projection.weight"))
    return z * torch.sigmoid(linear(x, P("gating_linear.weight")))


def grid_self_attention(pair, mask, params, transpose, num_head=4, prefix="", batch_chunk=64):
    """GridSelfAttention.forward / _attention_torch (xfold/nn/attention.py:61-78, 80-105).

    x = LN(pair); bias = (x W_b^T).permute(2, 0, 1) computed before the
    optional transpose; q, k, v = x W^T split into heads; attention with the
    un-transposed pair mask [N, N] as a per-batch-row key mask (:100); output
    times sigmoid(x W_gate^T); output projection; transpose back."""
    P = lambda n: _p(params, prefix, n)
    x = layer_norm(pair, P("act_norm.weight"), P("act_norm.bias"))
    bias = linear(x, P("pair_bias_projection.weight")).permute(2, 0, 1)
    if transpose:
        x = x.permute(1, 0, 2)
    n_b, n_t, c = x.shape
    d = c // num_head

    def heads(t):
        return t.reshape(n_b, n_t, num_head, d).permute(0, 2, 1, 3)

    q = heads(linear(x, P("q_projection.weight")))
    k = heads(linear(x, P("k_projection.weight")))
    v = heads(linear(x, P("v_projection.weight")))
    o = dot_product_attention(q, k, v, mask=mask, bias=bias, query_chunk=batch_chunk)
    o = o.permute(0, 2, 1, 3).reshape(n_b, n_t, c)
    o = o * torch.sigmoid(linear(x, P("gating_query.weight")))
    out = linear(o, P("output_projection.weight"))
    if transpose:
        out = out.permute(1, 0, 2)
    return out


def _projected_channels(pair, mask, params, prefix, row_slice):
    """Rows `row_slice` of the masked, gated projection of
    triangle_multiplication (xfold/nn/triangle_multiplication.py:81-95):
    returns (a, b) as [c, rows, N] with a = channel 2c', b = channel 2c'+1."""
    P = lambda n: _p(params, prefix, n)
    x = layer_norm(pair[row_slice], P("left_norm_input.weight"), P("left_norm_input.bias"))
    proj = linear(x, P("projection.weight")).permute(2, 0, 1)
    if mask is not None:
        proj = proj * mask[row_slice][None, ...]
    proj = proj * torch.sigmoid(linear(x, P("gate.weight")).permute(2, 0, 1))
    c = pair.shape[-1]
    proj = proj.reshape(c, 2, *proj.shape[1:])
    return proj[:, 0], proj[:, 1]


def triangle_multiplication_rows(pair, mask, params, outgoing, rows, prefix="", chunk=128):
    """triangle_multiplication (above; xfold/nn/triangle_multiplication.py:71-105)
    evaluated only for the output rows `rows` (a list of indices i): returns
    update[rows] as [len(rows), N, c].  The projection of the whole pair is
    needed (all of b for outgoing, all of a for incoming) and is formed in
    slices of `chunk` pair rows; the contraction, centre LayerNorm, output
    projection and gate run for the selected rows only.  Same operations in
    the same order as the full function, so large pairs can be checked on a
    sample of rows."""
    P = lambda n: _p(params, prefix, n)
    n, _, c = pair.shape
    rows = list(rows)
    full = torch.empty(c, n, n, dtype=torch.float32)  # b (outgoing) or a (incoming)
    # outgoing: rows i of a, a[c, i, k]; incoming: columns i of b, b[c, k, i]
    sel = torch.empty(c, len(rows), n) if outgoing else torch.empty(c, n, len(rows))
    for r0 in range(0, n, chunk):
        r1 = min(n, r0 + chunk)
        a, b = _projected_channels(pair, mask, params, prefix, slice(r0, r1))
        full[:, r0:r1] = b if outgoing else a
        if outgoing:
            for s, i in enumerate(rows):
                if r0 <= i < r1:
                    sel[:, s] = a[:, i - r0]
        else:
            sel[:, r0:r1] = b[:, :, rows]
    if outgoing:
        z = torch.einsum("cik,cjk->cij", sel, full)
    else:
        z = torch.einsum("ckj,cki->cij", full, sel)
    z = z.permute(1, 2, 0)  # [R, N, c]
    z = layer_norm(z, P("center_norm.weight"), P("center_norm.bias"))
    z = linear(z, P("output_projection.weight"))
    x_rows = layer_norm(pair[rows], P("left_norm_input.weight"), P("left_norm_input.bias"))
    return z * torch.sigmoid(linear(x_rows, P("gating_linear.weight")))


def grid_self_attention_rows(pair, mask, params, transpose, rows, num_head=4, prefix="",
                             chunk=128):
    """grid_self_attention (above; xfold/nn/attention.py:61-105) evaluated only
    for the batch rows `rows`: pair rows i for the starting node (returns
    update[rows] as [R, N, c]) or pair columns j for the ending node (returns
    update[:, rows] transposed, i.e. [R, N, c] with element [r, i] = update[i,
    rows[r]]).  The bias of the whole pair (projected before the transpose,
    :87-98) is formed in slices of `chunk` rows; the key mask of batch row b is
    pair_mask[b] in both directions (:100)."""
    P = lambda n: _p(params, prefix, n)
    n, _, c = pair.shape
    d = c // num_head
    bias = torch.empty(num_head, n, n, dtype=torch.float32)
    for r0 in range(0, n, chunk):
        xs = layer_norm(pair[r0:r0 + chunk], P("act_norm.weight"), P("act_norm.bias"))
        bias[:, r0:r0 + xs.shape[0]] = linear(xs, P("pair_bias_projection.weight")).permute(2, 0, 1)
    outs = []
    for r in rows:
        src = pair[:, r] if transpose else pair[r]  # [N tokens, c]
        x = layer_norm(src, P("act_norm.weight"), P("act_norm.bias"))

        def heads(t):
            return t.reshape(1, n, num_head, d).permute(0, 2, 1, 3)

        q = heads(linear(x, P("q_projection.weight")))
        k = heads(linear(x, P("k_projection.weight")))
        v = heads(linear(x, P("v_projection.weight")))
        m = None if mask is None else mask[r:r + 1]
        o = dot_product_attention(q, k, v, mask=m, bias=bias)
        o = o.permute(0, 2, 1, 3).reshape(n, c)
        o = o * torch.sigmoid(linear(x, P("gating_query.weight")))
        outs.append(linear(o, P("output_projection.weight")))
    return torch.stack(outs, dim=0)


def transition(x, params, prefix=""):
    """Transition.forward (xfold/nn/primitives.py:33-37): LN -> GLU with
    transition1.weight.T -> transition2."""
    P = lambda n: _p(params, prefix, n)
    y = layer_norm(x, P("input_layer_norm.weight"), P("input_layer_norm.bias"))
    h = gated_linear_unit(y, P("transition1.weight").T)
    return linear(h, P("transition2.weight"))


def adaptive_layer_norm(x, single_cond, params, use_single_cond, prefix=""):
    """AdaptiveLayerNorm.forward (xfold/nn/diffusion_transformer.py:51-64)."""
    P = lambda n: _p(params, prefix, n)
    if use_single_cond:
        x = layer_norm(x)
        sc = layer_norm(single_cond, P("single_cond_layer_norm.weight"), None)
        scale = linear(sc, P("single_cond_scale.weight"), P("single_cond_scale.bias"))
        shift = linear(sc, P("single_cond_bias.weight"))
        return torch.sigmoid(scale) * x + shift
    return layer_norm(x, P("layer_norm.weight"), P("layer_norm.bias"))


def ada_ln_zero(x, single_cond, params, use_single_cond, prefix=""):
    """AdaLNZero.forward (xfold/nn/diffusion_transformer.py:85-95)."""
    P = lambda n: _p(params, prefix, n)
    out = linear(x, P("transition2.weight"))
    if use_single_cond:
        cond = linear(single_cond, P("adaptive_zero_cond.weight"), P("adaptive_zero_cond.bias"))
        out = torch.sigmoid(cond) * out
    return out


def self_attention(x, mask, pair_logits, params, single_cond=None, num_head=16,
                   use_single_cond=False, prefix=""):
    """SelfAttention._forward_torch (xfold/nn/diffusion_transformer.py:184-217)."""
    P = lambda n: _p(params, prefix, n)
    y = adaptive_layer_norm(x, single_cond, params, use_single_cond, prefix + "adaptive_layernorm.")
    n, c = y.shape
    d = c // num_head

    def heads(t):
        return t.reshape(n, num_head, d).permute(1, 0, 2).unsqueeze(0)

    q = heads(linear(y, P("q_projection.weight"), P("q_projection.bias")))
    k = heads(linear(y, P("k_projection.weight")))
    v = heads(linear(y, P("v_projection.weight")))
    o = dot_product_attention(q, k, v, mask=mask, bias=pair_logits)
    o = o.squeeze(0).permute(1, 0, 2).reshape(n, c)
    o = o * torch.sigmoid(linear(y, P("gating_query.weight")))
    return ada_ln_zero(o, single_cond, params, use_single_cond, prefix + "adaptive_zero_init.")


def diffusion_transition(x, single_cond, params, use_single_cond=True, prefix=""):
    """DiffusionTransition.forward (xfold/nn/diffusion_transformer.py:124-128)."""
    P = lambda n: _p(params, prefix, n)
    y = adaptive_layer_norm(x, single_cond, params, use_single_cond, prefix + "adaptive_layernorm.")
    h = gated_linear_unit(y, P("transition1.weight").T)
    return ada_ln_zero(h, single_cond, params, use_single_cond, prefix + "adaptive_zero_init.")


def diffusion_transformer(act, mask, single_cond, pair_cond, params, num_blocks=24,
                          super_block_size=4, num_head=16, prefix=""):
    """DiffusionTransformer.forward (xfold/nn/diffusion_transformer.py:250-272):
    LN(pair_cond) once; per super-block the pair-logit projection rearranged
    'n s (b h) -> b h n s' (:262-265); then per block act += SelfAttention(act,
    mask, logits[j], single_cond) and act += DiffusionTransition(act,
    single_cond), both conditioned.  Returns a new tensor."""
    P = lambda n: _p(params, prefix, n)
    act = act.clone()
    pair_act = layer_norm(pair_cond, P("pair_input_layer_norm.weight"),
                          P("pair_input_layer_norm.bias"))
    n, s = pair_act.shape[:2]
    for sb in range(num_blocks // super_block_size):
        logits = linear(pair_act, P(f"pair_logits_projection.{sb}.weight"))
        logits = logits.reshape(n, s, super_block_size, num_head).permute(2, 3, 0, 1)
        for j in range(super_block_size):
            i = sb * super_block_size + j
            act += self_attention(act, mask, logits[j], params, single_cond, num_head, True,
                                  prefix + f"self_attention.{i}.")
            act += diffusion_transition(act, single_cond, params, True,
                                        prefix + f"transition_block.{i}.")
    return act


def pair_logits(pair, params, prefix=""):
    """Single-track pair logits (xfold/nn/pairformer.py:103-106): LN then a
    bias-free projection to heads, permuted to [H, N, N]."""
    P = lambda n: _p(params, prefix, n)
    x = layer_norm(pair, P("single_pair_logits_norm.weight"), P("single_pair_logits_norm.bias"))
    return linear(x, P("single_pair_logits_projection.weight")).permute(2, 0, 1)


def atom_layout_convert(gather_idxs, gather_mask, arr):
    """atom_layout.convert with layout_axes=(-3, -2) (xfold/nn/atom_layout.py:88-160)
    for arr [A, B, c]: flatten the two layout axes, gather rows by gather_idxs,
    zero rows whose gather_mask is False."""
    flat = arr.reshape(-1, arr.shape[-1])
    out = flat[gather_idxs.long()]
    return out * gather_mask.to(out.dtype)[..., None]


def cross_attention(x_q, x_k, mask_q, mask_k, pair_logits, params, single_cond_q, single_cond_k,
                    num_head=4, prefix=""):
    """CrossAttention.forward (xfold/nn/diffusion_transformer.py:307-350) on
    [subsets, queries, c] / [subsets, keys, c]: AdaLN of both sides, the
    reference's bias 1e9 * !mask_q[q] * !mask_k[k] (:318-322) added to the
    scaled logits before the pair logits (:336-340), softmax, gate, AdaLNZero."""
    P = lambda n: _p(params, prefix, n)
    bias = 1e9 * mask_q.logical_not()[..., None, :, None] * mask_k.logical_not()[..., None, None, :]
    xq = adaptive_layer_norm(x_q, single_cond_q, params, True, prefix + "q_adaptive_layernorm.")
    xk = adaptive_layer_norm(x_k, single_cond_k, params, True, prefix + "k_adaptive_layernorm.")
    c = xq.shape[-1]
    d = c // num_head
    q = linear(xq, P("q_projection.weight"), P("q_projection.bias"))
    k = linear(xk, P("k_projection.weight"))
    q = q.reshape(q.shape[:-1] + (num_head, d))
    k = k.reshape(k.shape[:-1] + (num_head, d))
    logits = torch.einsum("...qhc,...khc->...hqk", q * d ** (-0.5), k) + bias
    if pair_logits is not None:
        logits = logits + pair_logits
    weights = torch.softmax(logits, dim=-1)
    v = linear(xk, P("v_projection.weight"))
    v = v.reshape(v.shape[:-1] + (num_head, d))
    o = torch.einsum("...hqk,...khc->...qhc", weights, v)
    o = o.reshape(o.shape[:-2] + (-1,))
    o = o * torch.sigmoid(linear(xq, P("gating_query.weight")))
    return ada_ln_zero(o, single_cond_q, params, True, prefix + "adaptive_zero_init.")


def cross_pair_logits(pair_cond, params, num_blocks=3, num_head=4, prefix=""):
    """The cached pair logits of DiffusionCrossAttTransformer
    (xfold/nn/diffusion_transformer.py:376-380): LN (weight only) then the
    projection, rearranged 'n q k (b h) -> b n h q k'."""
    P = lambda n: _p(params, prefix, n)
    x = layer_norm(pair_cond, P("pair_input_layer_norm.weight"), None)
    y = linear(x, P("pair_logits_projection.weight"))  # [n, q, k, b*h]
    s, nq, nk, _ = y.shape
    return y.reshape(s, nq, nk, num_blocks, num_head).permute(3, 0, 4, 1, 2)


def diffusion_cross_att_transformer(queries_act, queries_mask, gather_idxs, gather_mask,
                                    keys_mask, queries_single_cond, keys_single_cond, pair_cond,
                                    params, num_blocks=3, num_head=4, prefix="", logits=None):
    """DiffusionCrossAttTransformer.forward (xfold/nn/diffusion_transformer.py:382-411):
    per block, keys gathered from the current queries, then the cross-attention
    and the conditioned transition updates.  Returns the new queries_act.
    `logits` passes the pair logits the reference holds in its input cache."""
    if logits is None:
        logits = cross_pair_logits(pair_cond, params, num_blocks, num_head, prefix)
    act = queries_act.clone()
    for i in range(num_blocks):
        keys = atom_layout_convert(gather_idxs, gather_mask, act)
        act = act + cross_attention(act, keys, queries_mask, keys_mask, logits[i], params,
                                    queries_single_cond, keys_single_cond, num_head,
                                    f"{prefix}cross_attention.{i}.")
        act = act + diffusion_transition(act, queries_single_cond, params, True,
                                         f"{prefix}transition_block.{i}.")
    return act


def msa_attention(msa, msa_mask, pair, params, num_head=8, prefix=""):
    """MSAAttention.forward (xfold/nn/attention.py:125-144): softmax over keys
    of the pair logits plus 1e9 (max over sequences of msa_mask - 1), shared by
    every MSA row; per-head weighted average of v, sigmoid gate, output
    projection."""
    P = lambda n: _p(params, prefix, n)
    x = layer_norm(msa, P("act_norm.weight"), P("act_norm.bias"))
    p = layer_norm(pair, P("pair_norm.weight"), P("pair_norm.bias"))
    logits = linear(p, P("pair_logits.weight")).permute(2, 0, 1)
    logits = logits + 1e9 * (torch.max(msa_mask, dim=0).values - 1.0)
    weights = torch.softmax(logits, dim=-1)
    v = linear(x, P("v_projection.weight"))
    v = v.reshape(v.shape[:-1] + (num_head, -1))
    o = torch.einsum("hqk,bkhc->bqhc", weights, v)
    o = o.reshape(o.shape[:-2] + (-1,))
    o = o * torch.sigmoid(linear(x, P("gating_query.weight")))
    return linear(o, P("output_projection.weight"))


def outer_product_mean(msa, mask, params, prefix=""):
    """OuterProductMean.forward (xfold/nn/primitives.py:62-75): the masked left /
    right projections' outer product summed over sequences, contracted with
    output_w [c, e, f] plus output_b, divided by (1e-3 + the mask overlap
    count); returns the [N, N, f] pair update."""
    P = lambda n: _p(params, prefix, n)
    m = mask.unsqueeze(-1)
    x = layer_norm(msa, P("layer_norm_input.weight"), P("layer_norm_input.bias"))
    left = m * linear(x, P("left_projection.weight"))
    right = m * linear(x, P("right_projection.weight"))
    act = torch.einsum("aic,aje->icje", left, right)
    act = torch.einsum("icje,cef->ijf", act, P("output_w")) + P("output_b")
    norm = torch.einsum("ai,aj->ij", mask, mask)[..., None]
    return act / (1e-3 + norm)


def pairformer_block(pair, pair_mask, single, seq_mask, params, n_heads=16, n_heads_pair=4,
                     with_single=True, prefix=""):
    """PairformerBlock.forward (xfold/nn/pairformer.py:77-114): five in-place
    residual updates of pair, then (with_single) the single track.  Returns new
    tensors (inputs untouched)."""
    pair = pair.clone()
    pair += triangle_multiplication(pair, pair_mask, params, True,
                                    prefix + "triangle_multiplication_outgoing.")
    pair += triangle_multiplication(pair, pair_mask, params, False,
                                    prefix + "triangle_multiplication_incoming.")
    pair += grid_self_attention(pair, pair_mask, params, False, n_heads_pair,
                                prefix + "pair_attention1.")
    pair += grid_self_attention(pair, pair_mask, params, True, n_heads_pair,
                                prefix + "pair_attention2.")
    pair += transition(pair, params, prefix + "pair_transition.")
    if not with_single:
        return pair
    single = single.clone()
    logits = pair_logits(pair, params, prefix)
    single += self_attention(single, seq_mask, logits, params, None, n_heads, False,
                             prefix + "single_attention_.")
    single += transition(single, params, prefix + "single_transition.")
    return pair, single


def evoformer_block(msa, pair, msa_mask, pair_mask, params, n_heads_pair=4, prefix=""):
    """EvoformerBlock.forward (xfold/nn/pairformer.py:138-156): the outer
    product mean into pair, MSA attention and transition into msa, then the
    pair stack.  Returns new (msa, pair) tensors."""
    msa, pair = msa.clone(), pair.clone()
    pair += outer_product_mean(msa, msa_mask, params, prefix + "outer_product_mean.")
    msa += msa_attention(msa, msa_mask, pair, params, 8, prefix + "msa_attention1.")
    msa += transition(msa, params, prefix + "msa_transition.")
    pair = pairformer_block(pair, pair_mask, None, None, params, n_heads_pair=n_heads_pair,
                            with_single=False, prefix=prefix)
    return msa, pair


def evoformer_block_flops(s, n, c_msa=64, c_pair=128, heads_pair=4):
    """Algorithmic FLOPs of one Evoformer block: outer product mean (both
    contractions and the projections), MSA attention, MSA transition, and the
    pair stack of a Pairformer block."""
    sn = s * n
    opm = 2 * sn * c_msa * 64 + 2 * s * (32 * n) ** 2 + 2 * n * n * 1024 * c_pair
    msa_att = (2 * sn * c_msa * 128 + 2 * n * n * c_pair * 8 + 2 * 8 * n * n * s * 8
               + 2 * sn * 64 * 64)
    msa_tr = 2 * sn * c_msa * (8 * c_msa) + 2 * sn * (4 * c_msa) * c_msa
    f = pairformer_block_flops(n, c_pair, 384, heads_pair, 16)
    pair_stack = f["triangle_multiplication"] + f["triangle_attention"] + f["pair_transition"]
    return {"outer_product_mean": opm, "msa_attention": msa_att, "msa_transition": msa_tr,
            "pair": pair_stack, "total": opm + msa_att + msa_tr + pair_stack}


# --------------------------------------------------------------------------- FLOP counts

def pairformer_block_flops(n, c_pair=128, c_single=384, heads_pair=4, heads_single=16):
    """Algorithmic FLOPs of one Pairformer block (multiply-add = 2)."""
    n2 = n * n
    tri = 2 * (2 * n2 * c_pair * (4 * c_pair + c_pair) + 2 * c_pair * n ** 3 + 2 * n2 * c_pair * c_pair)
    d = c_pair // heads_pair
    att = 2 * (2 * n2 * c_pair * (4 * c_pair + heads_pair) + 4 * heads_pair * n ** 3 * d
               + 2 * n2 * c_pair * c_pair)
    glu = 2 * n2 * c_pair * 8 * c_pair + 2 * n2 * 4 * c_pair * c_pair
    ds = c_single // heads_single
    single = (2 * n2 * c_pair * heads_single + 2 * n * c_single * 5 * c_single
              + 4 * heads_single * n2 * ds + 2 * n * c_single * 8 * c_single
              + 2 * n * 4 * c_single * c_single)
    return {"triangle_multiplication": tri, "triangle_attention": att, "pair_transition": glu,
            "single_track": single, "total": tri + att + glu + single}


def triangle_multiplication_flops(n, c=128):
    return 2 * n * n * c * 5 * c + 2 * c * n ** 3 + 2 * n * n * c * c


def triangle_attention_flops(n, c=128, heads=4):
    d = c // heads
    return 2 * n * n * c * (4 * c + heads) + 4 * heads * n ** 3 * d + 2 * n * n * c * c


def relative_error(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max|got - ref| / max|ref| in float64 (the parity metric of the tests)."""
    got = got.detach().to("cpu", torch.float64)
    ref = ref.detach().to("cpu", torch.float64)
    denom = ref.abs().max().item()
    if denom == 0.0:
        return (got - ref).abs().max().item()
    return (got - ref).abs().max().item() / denom


__all__ = [name for name in dir() if not name.startswith("_") and name not in ("math", "torch", "F")]
