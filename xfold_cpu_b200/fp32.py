"""float32 compute path of the hot-path operators.

The `cuda` backend computes in bf16 on the tensor cores, like the reference's
GPU route (autocast bf16).  With `fastnn.config.compute_dtype = "float32"` the
modules instead run these functions: the reference's float32 route (no
autocast, xfold/fastnn/native.py:31-43) restated on the library's fp32 CUDA-core
kernels (xfb_f32_gemm / _layer_norm / _attention / _silu_mul / _scale_shift),
matching the reference torch path to ~1e-6 (contract: 1e-4).  Every reshape,
permute, head split and the triangle multiplication's channel interleave is a
strided view handed to the kernels; nothing here computes on the CPU, and a
missing library raises RuntimeError like the bf16 path.
"""

from __future__ import annotations

import ctypes

import torch

from . import _capi


def _f32(t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("the float32 path takes CUDA tensors")
    return t if t.dtype == torch.float32 else t.float()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, bias=None, act: int = 0,
         row_scale=None, mul=None, accumulate: bool = False) -> torch.Tensor:
    """out[bt](i, j) (=|+=) ((act(sum_k a[bt](i, k) b[bt](j, k) + bias[j])) * row_scale[bt](i))
    * mul[bt](i, j) for 3-D (batched) views of any strides; act 1 = sigmoid.
    row_scale is [batch, M] (or a view of it), mul [batch, M, N]."""
    a, b, bias, row_scale, mul = (_f32(t) for t in (a, b, bias, row_scale, mul))
    if out.dtype != torch.float32 or not out.is_cuda:
        raise ValueError("out must be a float32 CUDA tensor")
    batch, m, k = a.shape
    n = b.shape[1]
    if b.shape != (batch, n, k) and b.shape != (1, n, k):
        raise ValueError(f"gemm operand shapes {tuple(a.shape)} / {tuple(b.shape)} differ")
    if out.shape != (batch, m, n):
        raise ValueError("gemm output shape mismatch")
    if bias is not None:
        bias = bias.contiguous()
    args = _capi.F32GemmArgs()
    args.a, (args.a_sb, args.a_si, args.a_sk) = a.data_ptr(), a.stride()
    args.b = b.data_ptr()
    args.b_sb = 0 if b.shape[0] == 1 else b.stride(0)
    args.b_sj, args.b_sk = b.stride(1), b.stride(2)
    args.c, (args.c_sb, args.c_si, args.c_sj) = out.data_ptr(), out.stride()
    args.m, args.n, args.k, args.batch = m, n, k, batch
    args.bias = _ptr(bias)
    args.act = act
    if row_scale is not None:
        args.row_scale, (args.rs_sb, args.rs_si) = row_scale.data_ptr(), row_scale.stride()
    if mul is not None:
        args.mul, (args.mul_sb, args.mul_si, args.mul_sj) = mul.data_ptr(), mul.stride()
    args.accumulate = int(accumulate)
    _capi.call("xfb_f32_gemm", ctypes.addressof(args), _stream(out))
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias=None, act: int = 0, mul=None,
           out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """x [..., K] @ weight[N, K]^T (+ bias), optional sigmoid and product with
    `mul` [..., N]; x may be any strided view whose last dim has stride 1 or not."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if out is None:
        out = torch.empty((*lead, weight.shape[0]), dtype=torch.float32, device=x.device)
    o2 = out.view(-1, weight.shape[0])
    m2 = None if mul is None else _f32(mul).reshape(-1, weight.shape[0])
    gemm(x2.unsqueeze(0), _f32(weight).unsqueeze(0), o2.unsqueeze(0), bias=bias, act=act,
         mul=None if m2 is None else m2.unsqueeze(0), accumulate=accumulate)
    return out


def layer_norm(x: torch.Tensor, weight=None, bias=None, eps: float = 1e-5) -> torch.Tensor:
    x = _f32(x).contiguous()
    c = x.shape[-1]
    y = torch.empty_like(x)
    _capi.call("xfb_f32_layer_norm", x.data_ptr(), x.numel() // c, c, c, _ptr(_f32(weight)),
               _ptr(_f32(bias)), float(eps), y.data_ptr(), c, _stream(x))
    return y


def attention(q, k, v, out, bias=None, mask=None, gate=None, scale=None) -> torch.Tensor:
    """out = gate * softmax(q k^T * scale + bias, mask) v on 4-D [B, H, n, d]
    views (last dim contiguous); bias broadcastable to [B, H, Q, K] with a
    contiguous key dim; mask [B or 1, K] (0 = masked)."""
    q, k, v, bias, mask, gate = (_f32(t) for t in (q, k, v, bias, mask, gate))
    bsz, h, nq, d = q.shape
    nk, dv = k.shape[2], v.shape[3]
    for t in (q, k, v, out) + ((gate,) if gate is not None else ()):
        if t.stride(-1) != 1:
            raise ValueError("attention rows must be contiguous in the head dimension")
    args = _capi.F32AttentionArgs()
    args.q, (args.q_sb, args.q_sh, args.q_si, _) = q.data_ptr(), q.stride()
    args.k, (args.k_sb, args.k_sh, args.k_si, _) = k.data_ptr(), k.stride()
    args.v, (args.v_sb, args.v_sh, args.v_si, _) = v.data_ptr(), v.stride()
    if bias is not None:
        bias = bias.expand(bsz, h, nq, nk)
        if bias.stride(-1) != 1:
            bias = bias.contiguous()
        args.bias, (args.bias_sb, args.bias_sh, args.bias_si, _) = bias.data_ptr(), bias.stride()
    if mask is not None:
        if mask.dim() > 2:
            if mask.dim() != 4 or mask.shape[1] != 1 or mask.shape[2] != 1:
                raise ValueError("the float32 attention takes key masks [K], [B, K] or "
                                 "[B, 1, 1, K]")
        mask = mask.reshape(-1, nk)
        if mask.shape[0] not in (1, bsz):
            raise ValueError("mask batch must be 1 or the attention batch")
        if mask.stride(-1) != 1:
            mask = mask.contiguous()
        args.mask = mask.data_ptr()
        args.mask_sb = 0 if mask.shape[0] == 1 else mask.stride(0)
    args.out, (args.out_sb, args.out_sh, args.out_si, _) = out.data_ptr(), out.stride()
    if gate is not None:
        args.gate, (args.gate_sb, args.gate_sh, args.gate_si, _) = gate.data_ptr(), gate.stride()
    args.batch, args.heads, args.nq, args.nk, args.d, args.dv = bsz, h, nq, nk, d, dv
    args.scale = d ** -0.5 if scale is None else float(scale)
    _capi.call("xfb_f32_attention", ctypes.addressof(args), _stream(out))
    return out


def silu_mul(h: torch.Tensor) -> torch.Tensor:
    h = _f32(h).contiguous()
    f = h.shape[-1] // 2
    y = torch.empty((*h.shape[:-1], f), dtype=torch.float32, device=h.device)
    _capi.call("xfb_f32_silu_mul", h.data_ptr(), h.numel() // (2 * f), f, y.data_ptr(),
               _stream(h))
    return y


def scale_shift_(y: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    scale, shift = _f32(scale).contiguous(), _f32(shift).contiguous()
    if not y.is_contiguous() or scale.shape != y.shape or shift.shape != y.shape:
        raise ValueError("scale_shift_ takes contiguous tensors of one shape")
    _capi.call("xfb_f32_scale_shift", y.data_ptr(), scale.data_ptr(), shift.data_ptr(),
               y.numel(), _stream(y))
    return y


# ----------------------------------------------------------------------------- operators

def triangle_multiplication(mod, pair: torch.Tensor, mask: torch.Tensor | None) -> torch.Tensor:
    """TriangleMultiplication._forward_torch (triangle_multiplication.py:71-105)
    in fp32: returns the update [N, N, c]."""
    n, _, c = pair.shape
    dev = pair.device
    x = layer_norm(pair, mod.left_norm_input.weight, mod.left_norm_input.bias,
                   mod.left_norm_input.eps)
    g = linear(x, mod.gate.weight, act=1)                               # sigmoid(gate) [N, N, 2c]
    p = torch.empty((n, n, 2 * c), dtype=torch.float32, device=dev)
    rs = None if mask is None else _f32(mask).reshape(1, n * n).contiguous()
    gemm(x.view(1, n * n, c), _f32(mod.projection.weight).unsqueeze(0), p.view(1, n * n, 2 * c),
         row_scale=rs, mul=g.view(1, n * n, 2 * c))                      # proj * mask * gate
    pv = p.view(n, n, c, 2)
    a = pv[..., 0].permute(2, 0, 1)                                      # a[c, i, k] = p[i, k, 2c]
    b = pv[..., 1].permute(2, 0, 1)
    z = torch.empty((n, n, c), dtype=torch.float32, device=dev)
    zc = z.permute(2, 0, 1)                                              # z[c, i, j] in [i, j, c]
    if mod.equation == "cik,cjk->cij":
        gemm(a, b, zc)
    else:                                                                # 'ckj,cki->cij'
        gemm(b.transpose(1, 2), a.transpose(1, 2), zc)
    y = layer_norm(z, mod.center_norm.weight, mod.center_norm.bias, mod.center_norm.eps)
    gl = linear(x, mod.gating_linear.weight, act=1)
    return linear(y, mod.output_projection.weight, mul=gl)


def grid_self_attention(mod, pair: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """GridSelfAttention.forward (attention.py:80-105) in fp32: the bias from the
    un-transposed LayerNorm'd pair, attention over rows of the (transposed)
    pair with the un-transposed mask rows, the update transposed back."""
    n, _, c = pair.shape
    h = mod.num_head
    d = c // h
    dev = pair.device
    x = layer_norm(pair, mod.act_norm.weight, mod.act_norm.bias, mod.act_norm.eps)
    bias = torch.empty((h, n, n), dtype=torch.float32, device=dev)
    gemm(x.view(1, n * n, c), _f32(mod.pair_bias_projection.weight).unsqueeze(0),
         bias.view(h, n * n).t().unsqueeze(0))                           # bias[h, q, k]
    xs = x.transpose(0, 1) if mod.transpose else x                       # [b, i, c] view

    def proj(weight, act=0):
        t = torch.empty((n, n, c), dtype=torch.float32, device=dev)
        gemm(xs, _f32(weight).unsqueeze(0), t, act=act)
        return t

    q, k, v = (proj(w) for w in (mod.q_projection.weight, mod.k_projection.weight,
                                 mod.v_projection.weight))
    gate = proj(mod.gating_query.weight, act=1)

    def heads(t):
        return t.view(n, n, h, d).permute(0, 2, 1, 3)                   # [b, h, i, d]

    o = torch.empty((n, n, c), dtype=torch.float32, device=dev)
    attention(heads(q), heads(k), heads(v), heads(o), bias=bias.unsqueeze(0), mask=mask,
              gate=heads(gate))
    upd = torch.empty((n, n, c), dtype=torch.float32, device=dev)
    target = upd.transpose(0, 1) if mod.transpose else upd
    gemm(o, _f32(mod.output_projection.weight).unsqueeze(0), target)
    return upd


def transition(mod, x: torch.Tensor) -> torch.Tensor:
    """Transition.forward (primitives.py:33-37): LN, GLU (first half the SiLU
    gate), output projection."""
    y = layer_norm(x, mod.input_layer_norm.weight, mod.input_layer_norm.bias,
                   mod.input_layer_norm.eps)
    hcat = linear(y, mod.transition1.weight)
    return linear(silu_mul(hcat), mod.transition2.weight)


def adaptive_layer_norm(ada, x: torch.Tensor, single_cond=None) -> torch.Tensor:
    """AdaptiveLayerNorm.forward (diffusion_transformer.py:51-64)."""
    ln = ada.layer_norm
    y = layer_norm(x, ln.weight, ln.bias, ln.eps)
    if not ada.use_single_cond:
        return y
    sc = layer_norm(single_cond, ada.single_cond_layer_norm.weight, None,
                    ada.single_cond_layer_norm.eps)
    scale = linear(sc, ada.single_cond_scale.weight, ada.single_cond_scale.bias, act=1)
    shift = linear(sc, ada.single_cond_bias.weight)
    return scale_shift_(y, scale, shift)


def ada_ln_zero(zero, x: torch.Tensor, single_cond=None) -> torch.Tensor:
    """AdaLNZero.forward (diffusion_transformer.py:85-95)."""
    if not zero.use_single_cond:
        return linear(x, zero.transition2.weight)
    cond = linear(single_cond, zero.adaptive_zero_cond.weight, zero.adaptive_zero_cond.bias, act=1)
    return linear(x, zero.transition2.weight, mul=cond)


def self_attention(mod, x: torch.Tensor, mask=None, pair_logits=None, single_cond=None):
    """SelfAttention._forward_torch (diffusion_transformer.py:184-217) in fp32."""
    n, c = x.shape
    h = mod.num_head
    d = c // h
    y = adaptive_layer_norm(mod.adaptive_layernorm, x, single_cond)
    q = linear(y, mod.q_projection.weight, mod.q_projection.bias)
    k = linear(y, mod.k_projection.weight)
    v = linear(y, mod.v_projection.weight)
    gate = linear(y, mod.gating_query.weight, act=1)

    def heads(t):
        return t.view(1, n, h, d).permute(0, 2, 1, 3)

    o = torch.empty((n, c), dtype=torch.float32, device=x.device)
    attention(heads(q), heads(k), heads(v), heads(o),
              bias=None if pair_logits is None else _f32(pair_logits).unsqueeze(0),
              mask=None if mask is None else _f32(mask).reshape(1, n), gate=heads(gate))
    return ada_ln_zero(mod.adaptive_zero_init, o, single_cond)


def diffusion_transition(mod, x: torch.Tensor, single_cond=None) -> torch.Tensor:
    """DiffusionTransition.forward (diffusion_transformer.py:124-128)."""
    y = adaptive_layer_norm(mod.adaptive_layernorm, x, single_cond)
    hcat = linear(y, mod.transition1.weight)
    return ada_ln_zero(mod.adaptive_zero_init, silu_mul(hcat), single_cond)


def pair_logits(block, pair: torch.Tensor) -> torch.Tensor:
    """[H, N, N] single-attention logits (pairformer.py:103-106)."""
    n, _, c = pair.shape
    norm = block.single_pair_logits_norm
    x = layer_norm(pair, norm.weight, norm.bias, norm.eps)
    w = block.single_pair_logits_projection.weight
    out = torch.empty((w.shape[0], n, n), dtype=torch.float32, device=pair.device)
    gemm(x.view(1, n * n, c), _f32(w).unsqueeze(0), out.view(w.shape[0], n * n).t().unsqueeze(0))
    return out


def pairformer_block(block, pair, pair_mask, single=None, seq_mask=None):
    """PairformerBlock.forward (pairformer.py:77-114) in fp32, in place on the
    f32 pair (and single)."""
    pair += triangle_multiplication(block.triangle_multiplication_outgoing, pair, pair_mask)
    pair += triangle_multiplication(block.triangle_multiplication_incoming, pair, pair_mask)
    pair += grid_self_attention(block.pair_attention1, pair, pair_mask)
    pair += grid_self_attention(block.pair_attention2, pair, pair_mask)
    pair += transition(block.pair_transition, pair)
    if not block.with_single:
        return pair
    logits = pair_logits(block, pair)
    single += self_attention(block.single_attention_, single, seq_mask, logits)
    single += transition(block.single_transition, single)
    return pair, single
