"""Torch-facing wrappers of the C ABI, one per operator of af3_kernels._C.

Mirrors af3_kernels/src/af3_kernels/__init__.py (lazy loader + wrappers) and
the pybind signatures of af3_kernels/src/csrc/bindings.cpp:10-49, with CUDA
tensors instead of CPU tensors:

    triangle_multiplication, dot_product_attention, gated_linear_unit, linear,
    layer_norm, runtime_info

plus the fused module-level operators grid_self_attention, transition,
self_attention and pair_logits.  Tensors must live on one sm_100 device;
weights are bf16 in nn.Linear layout [out, in] (see prepare_weight).  Work is
enqueued on torch's current stream; nothing synchronises.  Scratch comes from
torch's caching allocator and is released when the call returns.

Errors: shape / dtype problems raise ValueError (the reference raises
RuntimeError from TORCH_CHECK for the same cases, ValueError from its Python
bridges); CUDA failures raise RuntimeError.
"""

from __future__ import annotations

import torch

from . import _capi

_DTYPE_CODE = {torch.float32: _capi.F32, torch.bfloat16: _capi.BF16, torch.uint8: _capi.U8,
               torch.bool: _capi.U8}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError as error:
        raise ValueError(f"unsupported dtype {t.dtype}") from error


def _check_cuda(*tensors: torch.Tensor | None) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("the cuda backend requires CUDA tensors")
        if t.layout != torch.strided:
            raise ValueError("the cuda backend requires strided tensors")
        if torch.is_grad_enabled() and t.requires_grad:
            raise RuntimeError("the cuda backend supports inference only; disable gradients")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("all tensors must be on the same device")
    if device is None:
        raise ValueError("no tensor given")
    return device


def _contig(t: torch.Tensor | None, dtype: torch.dtype | None = None) -> torch.Tensor | None:
    if t is None:
        return None
    t = t.detach()
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def runtime_info() -> dict:
    """Build and device description (af3_kernels runtime_info, bindings.cpp:13-20)."""
    return _capi.runtime_info()


def check_device(device: torch.device | int | None = None) -> None:
    """Preflight for the cuda backend: sm_100 device and loadable kernels."""
    if not torch.cuda.is_available():
        raise ValueError("the cuda backend requires a CUDA device")
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        _capi.call("xfb_check_device")


def prepare_weight(weight: torch.Tensor) -> torch.Tensor:
    """bf16 contiguous copy of an nn.Linear weight [out, in] (no transpose)."""
    return _contig(weight, torch.bfloat16)


# ----------------------------------------------------------------------------- primitives

def layer_norm(x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None,
               eps: float = 1e-5) -> torch.Tensor:
    """bf16 LayerNorm over the last dimension (f32 statistics)."""
    device = _check_cuda(x, weight, bias)
    x = _contig(x)
    cols = x.shape[-1]
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=device)
    w, b = _contig(weight, torch.float32), _contig(bias, torch.float32)
    _capi.call("xfb_layer_norm", _ptr(x), _code(x), x.numel() // max(cols, 1), cols, _ptr(w),
               _ptr(b), float(eps), _ptr(y), _stream(device))
    return y


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """x[..., k] @ weight[n, k]^T (+ bias) with bf16 inputs and f32 accumulation."""
    device = _check_cuda(x, weight, bias)
    x = _contig(x, torch.bfloat16)
    weight = prepare_weight(weight)
    k = x.shape[-1]
    n = weight.shape[0]
    if weight.shape[1] != k:
        raise ValueError("linear weight must be [out, in] with in == x.shape[-1]")
    y = torch.empty((*x.shape[:-1], n), dtype=out_dtype, device=device)
    b = _contig(bias, torch.float32)
    _capi.call("xfb_linear", _ptr(x), x.numel() // k, k, _ptr(weight), n, _ptr(b), _ptr(y),
               _code(y), 0, _stream(device))
    return y


def gemm(a: torch.Tensor, b: torch.Tensor, mn_major: bool = False,
         out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Batched bf16 GEMM (af3_kernels gemm, bindings.cpp:26).

    K-major (mn_major=False): a [B, m, k], b [B, n, k] -> a @ b^T.
    MN-major (mn_major=True): a [B, k, m], b [B, k, n] -> a^T @ b."""
    device = _check_cuda(a, b)
    a, b = _contig(a, torch.bfloat16), _contig(b, torch.bfloat16)
    if a.dim() != 3 or b.dim() != 3 or a.shape[0] != b.shape[0]:
        raise ValueError("gemm expects batched 3-D operands")
    batch = a.shape[0]
    if mn_major:
        k, m = a.shape[1:]
        n = b.shape[2]
        if b.shape[1] != k:
            raise ValueError("gemm reduction dimensions differ")
    else:
        m, k = a.shape[1:]
        n = b.shape[1]
        if b.shape[2] != k:
            raise ValueError("gemm reduction dimensions differ")
    c = torch.empty((batch, m, n), dtype=out_dtype, device=device)
    _capi.call("xfb_gemm", _ptr(a), _ptr(b), _ptr(c), batch, m, n, k, int(mn_major),
               int(mn_major), _code(c), _stream(device))
    return c


def pack_glu_weight(weight: torch.Tensor) -> torch.Tensor:
    """Packs transition1.weight [2n, k] for gated_linear_unit(weight_packed=True)."""
    device = _check_cuda(weight)
    weight = _contig(weight)
    n2, k = weight.shape
    packed = torch.empty((n2, k), dtype=torch.bfloat16, device=device)
    _capi.call("xfb_pack_glu_weight", _ptr(weight), _code(weight), n2 // 2, k, _ptr(packed),
               _stream(device))
    return packed


def gated_linear_unit(x: torch.Tensor, weight: torch.Tensor,
                      weight_packed: bool = False) -> torch.Tensor:
    """silu(x @ W[:n]^T) * (x @ W[n:]^T) for W = transition1.weight [2n, k]."""
    device = _check_cuda(x, weight)
    x = _contig(x, torch.bfloat16)
    weight = weight if weight_packed else prepare_weight(weight)
    k = x.shape[-1]
    n = weight.shape[0] // 2
    m = x.numel() // k
    y = torch.empty((*x.shape[:-1], n), dtype=torch.bfloat16, device=device)
    ws = _workspace(0 if weight_packed else _capi.load().xfb_gated_linear_unit_workspace(m, k, n),
                    device)
    _capi.call("xfb_gated_linear_unit", _ptr(x), m, k, _ptr(weight), n, 1 if weight_packed else 0,
               _ptr(y), _ptr(ws), ws.numel(), _stream(device))
    return y


# ----------------------------------------------------------------------------- triangle mult.

def pack_triangle_weights(projection: torch.Tensor, gate: torch.Tensor,
                          gating_linear: torch.Tensor) -> torch.Tensor:
    device = _check_cuda(projection, gate, gating_linear)
    c = projection.shape[1]
    tensors = [_contig(t, torch.bfloat16) for t in (projection, gate, gating_linear)]
    packed = torch.empty((5 * c, c), dtype=torch.bfloat16, device=device)
    _capi.call("xfb_pack_triangle_weights", *(_ptr(t) for t in tensors), _capi.BF16, c,
               _ptr(packed), _stream(device))
    return packed


def triangle_multiplication(pair: torch.Tensor, mask: torch.Tensor | None, outgoing: bool,
                            left_weight: torch.Tensor, left_bias: torch.Tensor | None,
                            projection: torch.Tensor | None, gate: torch.Tensor | None,
                            center_weight: torch.Tensor, center_bias: torch.Tensor | None,
                            output_weight: torch.Tensor, gating_weight: torch.Tensor | None,
                            left_eps: float = 1e-5, center_eps: float = 1e-5,
                            weights_packed: bool = False, packed: torch.Tensor | None = None,
                            out: torch.Tensor | None = None, accumulate: bool = False,
                            out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """TriangleMultiplication update (af3_kernels triangle_multiplication,
    triangle_multiplication.cpp:6-73).  Returns the update, or adds it into
    `out` (f32 [N, N, C]) when accumulate=True."""
    device = _check_cuda(pair, mask, left_weight, output_weight)
    if pair.dim() != 3 or pair.shape[0] != pair.shape[1]:
        raise ValueError("Triangle input must be [N, N, C].")
    n, _, c = pair.shape
    pair = _contig(pair)
    if mask is not None:
        mask = _contig(mask.expand(n, n) if mask.dim() <= 2 else mask, torch.float32)
    if weights_packed:
        if packed is None:
            raise ValueError("weights_packed=True needs the packed buffer")
    else:
        projection, gate, gating_weight = (prepare_weight(t) for t in (projection, gate, gating_weight))
    output_weight = prepare_weight(output_weight)
    if out is None:
        if accumulate:
            raise ValueError("accumulate=True needs an output tensor")
        out = torch.empty((n, n, c), dtype=out_dtype, device=device)
    lw, lb = _contig(left_weight, torch.float32), _contig(left_bias, torch.float32)
    cw, cb = _contig(center_weight, torch.float32), _contig(center_bias, torch.float32)
    ws = _workspace(_capi.load().xfb_triangle_multiplication_workspace(n, c), device)
    _capi.call("xfb_triangle_multiplication", _ptr(pair), _code(pair), n, c, _ptr(mask),
               1 if outgoing else 0, _ptr(lw), _ptr(lb), _ptr(projection), _ptr(gate), _ptr(cw),
               _ptr(cb), _ptr(output_weight), _ptr(gating_weight),
               float(left_eps), float(center_eps), 1 if weights_packed else 0, _ptr(packed),
               _ptr(out), _code(out), 1 if accumulate else 0, _ptr(ws), ws.numel(),
               _stream(device))
    return out


# ----------------------------------------------------------------------------- attention

def dot_product_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          mask: torch.Tensor | None = None, bias: torch.Tensor | None = None,
                          q_pre_scaled: bool = False,
                          query_block: int | None = None) -> torch.Tensor:
    """softmax(q k^T / sqrt(d) + bias, mask) v for q, k, v [B, H, Q/K, D] (af3_kernels
    dot_product_attention, dot_product_attention.cpp:110-174).

    mask: rank 1 [K] or rank 2 [B, K] (any dtype, nonzero = keep), or a bool
    tensor broadcastable to [B, 1, 1, K].  bias: broadcastable to [B, H, Q, K]
    with the B dimension either B or 1.  query_block: the reference's CPU tile
    size, passed through the af3_kernels-compatible entry point (validated,
    no effect on results)."""
    device = _check_cuda(q, k, v, mask, bias)
    for t in (q, k, v):
        if t.dim() != 4:
            raise ValueError("attention expects [B, H, Q/K, D] tensors")
    B, H, nq, d = q.shape
    nk = k.shape[2]
    if k.shape != (B, H, nk, d) or v.shape[:3] != (B, H, nk) or v.shape[3] != d:
        raise ValueError("attention q/k/v shapes do not match (d == dv required)")
    q, k, v = (_contig(t, torch.bfloat16) for t in (q, k, v))
    mask_t, mask_code, mask_batched = None, _capi.F32, 0
    if mask is not None:
        if mask.dim() == 1:
            mask_t = _contig(mask, torch.float32 if mask.is_floating_point() else torch.uint8)
        elif mask.dim() == 2:
            mask_t = _contig(mask.expand(B, nk), torch.float32 if mask.is_floating_point()
                             else torch.uint8)
            mask_batched = 1
        else:
            if mask.dtype != torch.bool:
                raise ValueError("Attention masks of rank 0/3/4 must be boolean, as in the "
                                 "PyTorch path.")
            m4 = mask.reshape((1,) * (4 - mask.dim()) + tuple(mask.shape)) if mask.dim() < 4 else mask
            if m4.shape[1] != 1 or m4.shape[2] != 1:
                raise ValueError("the cuda attention supports key masks broadcast over heads "
                                 "and queries only")
            mask_t = _contig(m4.expand(B, 1, 1, nk).reshape(B, nk), torch.uint8)
            mask_batched = 1
        mask_code = _code(mask_t)
    bias_t, bias_batched = None, 0
    if bias is not None:
        b4 = bias.reshape((1,) * (4 - bias.dim()) + tuple(bias.shape)) if bias.dim() < 4 else bias
        bias_batched = 1 if b4.shape[0] != 1 else 0
        full = (B if bias_batched else 1, H, nq, nk)
        b4 = b4.expand(full)
        bias_t = _contig(b4, torch.bfloat16 if b4.dtype == torch.bfloat16 else torch.float32)
    out = torch.empty((B, H, nq, d), dtype=torch.bfloat16, device=device)
    ws = _workspace(_capi.load().xfb_dot_product_attention_workspace(B, H, nq, nk, d), device)
    bias_code = _code(bias_t) if bias_t is not None else _capi.BF16
    if query_block is None:
        _capi.call("xfb_dot_product_attention", _ptr(q), _ptr(k), _ptr(v), B, H, nq, nk, d,
                   _ptr(mask_t), mask_code, mask_batched, _ptr(bias_t), bias_code, bias_batched,
                   1 if q_pre_scaled else 0, _ptr(out), _ptr(ws), ws.numel(), _stream(device))
    else:
        _capi.call("xfb_af3_dot_product_attention", _ptr(q), _ptr(k), _ptr(v), B, H, nq, nk, d,
                   _ptr(mask_t), mask_code, mask_batched, _ptr(bias_t), bias_code, bias_batched,
                   int(query_block), 1 if q_pre_scaled else 0, _ptr(out), _ptr(ws), ws.numel(),
                   _stream(device))
    return out


def pack_attention_weights(q_w: torch.Tensor, k_w: torch.Tensor, v_w: torch.Tensor,
                           gate_w: torch.Tensor) -> torch.Tensor:
    device = _check_cuda(q_w, k_w, v_w, gate_w)
    c = q_w.shape[1]
    tensors = [_contig(t, torch.bfloat16) for t in (q_w, k_w, v_w, gate_w)]
    packed = torch.empty((4 * c, c), dtype=torch.bfloat16, device=device)
    _capi.call("xfb_pack_attention_weights", *(_ptr(t) for t in tensors), _capi.BF16, c,
               _ptr(packed), _stream(device))
    return packed


def grid_self_attention(pair: torch.Tensor, mask: torch.Tensor | None, transpose: bool,
                        norm_weight: torch.Tensor | None, norm_bias: torch.Tensor | None,
                        eps: float, bias_weight: torch.Tensor, packed: torch.Tensor,
                        output_weight: torch.Tensor, num_head: int,
                        out: torch.Tensor | None = None, accumulate: bool = False,
                        out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """GridSelfAttention update (xfold/nn/attention.py:80-105); `packed` is
    pack_attention_weights(q, k, v, gating_query)."""
    device = _check_cuda(pair, mask, bias_weight, packed, output_weight)
    n, _, c = pair.shape
    pair = _contig(pair)
    if mask is not None:
        mask = _contig(mask.expand(n, n), torch.float32)
    if out is None:
        out = torch.empty((n, n, c), dtype=out_dtype, device=device)
    # Converted copies stay referenced until the launch is enqueued: a freed
    # temporary's block can be handed to the next temporary before the kernel runs.
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    bw, ow = prepare_weight(bias_weight), prepare_weight(output_weight)
    ws = _workspace(_capi.load().xfb_grid_self_attention_workspace(n, c, num_head), device)
    _capi.call("xfb_grid_self_attention", _ptr(pair), _code(pair), n, c, num_head, _ptr(mask),
               1 if transpose else 0, _ptr(nw), _ptr(nb), float(eps), _ptr(bw), None, None, None,
               None, _ptr(ow), 1, _ptr(packed), _ptr(out), _code(out), 1 if accumulate else 0,
               _ptr(ws), ws.numel(), _stream(device))
    return out


def transition(x: torch.Tensor, norm_weight: torch.Tensor | None,
               norm_bias: torch.Tensor | None, eps: float, w1_packed: torch.Tensor,
               w2: torch.Tensor, factor: int, mod_scale: torch.Tensor | None = None,
               mod_shift: torch.Tensor | None = None, out_gate: torch.Tensor | None = None,
               out: torch.Tensor | None = None, accumulate: bool = False,
               out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """GLU transition update (Transition / DiffusionTransition); w1_packed is
    pack_glu_weight(transition1.weight), w2 = transition2.weight."""
    device = _check_cuda(x, w1_packed, w2, mod_scale, mod_shift, out_gate)
    c = x.shape[-1]
    rows = x.numel() // c
    x = _contig(x)
    mod_scale, mod_shift, out_gate = (_contig(t, torch.bfloat16) for t in (mod_scale, mod_shift, out_gate))
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype, device=device)
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    w2 = prepare_weight(w2)
    ws = _workspace(_capi.load().xfb_transition_workspace(rows, c, factor), device)
    _capi.call("xfb_transition", _ptr(x), _code(x), rows, c, factor, _ptr(nw), _ptr(nb),
               float(eps), _ptr(mod_scale), _ptr(mod_shift), _ptr(w1_packed), 1, _ptr(w2),
               _ptr(out_gate), _ptr(out), _code(out), 1 if accumulate else 0, _ptr(ws),
               ws.numel(), _stream(device))
    return out


def self_attention(x: torch.Tensor, mask: torch.Tensor | None, pair_logits: torch.Tensor | None,
                   norm_weight: torch.Tensor | None, norm_bias: torch.Tensor | None, eps: float,
                   packed: torch.Tensor, q_bias: torch.Tensor | None, wo: torch.Tensor,
                   num_head: int, mod_scale: torch.Tensor | None = None,
                   mod_shift: torch.Tensor | None = None, out_gate: torch.Tensor | None = None,
                   out: torch.Tensor | None = None, accumulate: bool = False,
                   out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """SelfAttention with pair bias (xfold/nn/diffusion_transformer.py:184-217)."""
    device = _check_cuda(x, mask, pair_logits, packed, wo)
    n, c = x.shape
    x = _contig(x)
    if mask is not None:
        mask = _contig(mask.expand(n), torch.float32)
    if pair_logits is not None:
        pair_logits = _contig(pair_logits, torch.bfloat16)
    mod_scale, mod_shift, out_gate = (_contig(t, torch.bfloat16) for t in (mod_scale, mod_shift, out_gate))
    if out is None:
        out = torch.empty((n, c), dtype=out_dtype, device=device)
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    qb, wo = _contig(q_bias, torch.float32), prepare_weight(wo)
    ws = _workspace(_capi.load().xfb_self_attention_workspace(n, c, num_head), device)
    _capi.call("xfb_self_attention", _ptr(x), _code(x), n, c, num_head, _ptr(mask),
               _ptr(pair_logits), _ptr(nw), _ptr(nb), float(eps), _ptr(mod_scale),
               _ptr(mod_shift), None, _ptr(qb), None, None, None, 1, _ptr(packed), _ptr(wo),
               _ptr(out_gate), _ptr(out), _code(out), 1 if accumulate else 0, _ptr(ws),
               ws.numel(), _stream(device))
    return out


def pair_logits(pair: torch.Tensor, norm_weight: torch.Tensor | None,
                norm_bias: torch.Tensor | None, eps: float, weight: torch.Tensor) -> torch.Tensor:
    """[H, N, N] bf16 logits = LN(pair) @ weight^T, permuted (pairformer.py:103-106)."""
    device = _check_cuda(pair, weight)
    n, _, c = pair.shape
    heads = weight.shape[0]
    pair = _contig(pair)
    logits = torch.empty((heads, n, n), dtype=torch.bfloat16, device=device)
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    w = prepare_weight(weight)
    _capi.call("xfb_pair_logits", _ptr(pair), _code(pair), n, c, heads, _ptr(nw), _ptr(nb),
               float(eps), _ptr(w), _ptr(logits), _stream(device))
    return logits


# ----------------------------------------------------------------------------- row-block stages
# The operators above take the whole pair.  These run them on a block of pair
# rows and stop where a row-sharded pair exchanges data between GPUs
# (xfold_cpu_b200/sharded.py).  Every block has n % 8 == 0 columns.

def _rows_of(t: torch.Tensor, name: str) -> tuple[int, int, int]:
    if t.dim() != 3:
        raise ValueError(f"{name} must be a [rows, n, c] row block")
    rows, n, c = t.shape
    if n % 8:
        raise ValueError(f"{name}: row blocks need n % 8 == 0 columns")
    return rows, n, c


def triangle_projection(pair: torch.Tensor, mask: torch.Tensor | None,
                        left_weight: torch.Tensor, left_bias: torch.Tensor | None,
                        left_eps: float, packed: torch.Tensor):
    """TriMul stage 1 on pair rows [rows, n, c]: returns a, b channel-major
    [c, rows, n] bf16 (projection channels 2k / 2k+1, masked and gated) and the
    output gate g [rows, n, c] (triangle_multiplication.py:71-95)."""
    device = _check_cuda(pair, mask, left_weight, packed)
    rows, n, c = _rows_of(pair, "pair")
    pair = _contig(pair)
    if mask is not None:
        mask = _contig(mask.expand(rows, n), torch.float32)
    a = torch.empty((c, rows, n), dtype=torch.bfloat16, device=device)
    b = torch.empty_like(a)
    g = torch.empty((rows, n, c), dtype=torch.bfloat16, device=device)
    lw, lb = _contig(left_weight, torch.float32), _contig(left_bias, torch.float32)
    ws = _workspace(_capi.load().xfb_triangle_projection_workspace(rows, n, c), device)
    _capi.call("xfb_triangle_projection", _ptr(pair), _code(pair), rows, n, c, _ptr(mask),
               _ptr(lw), _ptr(lb), float(left_eps), _ptr(packed), _ptr(a), _ptr(b), _ptr(g),
               _ptr(ws), ws.numel(), _stream(device))
    return a, b, g


def triangle_contraction(a: torch.Tensor, b: torch.Tensor, outgoing: bool) -> torch.Tensor:
    """TriMul contraction of a channel shard, a and b [cs, n, n] channel-major:
    outgoing z[c,i,j] = sum_k a[c,i,k] b[c,j,k]; incoming sum_k a[c,k,j] b[c,k,i]
    (triangle_multiplication.py:34-36).  bf16 out, f32 accumulation."""
    if outgoing:
        return gemm(a, b, mn_major=False, out_dtype=torch.bfloat16)
    return gemm(b, a, mn_major=True, out_dtype=torch.bfloat16)


def triangle_output(z: torch.Tensor, g: torch.Tensor, center_weight: torch.Tensor,
                    center_bias: torch.Tensor | None, center_eps: float,
                    output_weight: torch.Tensor, out: torch.Tensor | None = None,
                    accumulate: bool = False, out_dtype: torch.dtype = torch.bfloat16):
    """TriMul stage 3 on a row block: z channel-major [c, rows, n] (the
    contraction for these rows), g from stage 1; returns (LN_c(z) W_o^T) * g, or
    adds it into f32 `out` [rows, n, c] (triangle_multiplication.py:96-105)."""
    device = _check_cuda(z, g, center_weight, output_weight)
    c, rows, n = z.shape
    z, g = _contig(z, torch.bfloat16), _contig(g, torch.bfloat16)
    if out is None:
        if accumulate:
            raise ValueError("accumulate=True needs an output tensor")
        out = torch.empty((rows, n, c), dtype=out_dtype, device=device)
    cw, cb = _contig(center_weight, torch.float32), _contig(center_bias, torch.float32)
    ow = prepare_weight(output_weight)
    ws = _workspace(_capi.load().xfb_triangle_output_workspace(rows, n, c), device)
    _capi.call("xfb_triangle_output", _ptr(z), rows, n, c, _ptr(g), _ptr(cw), _ptr(cb),
               float(center_eps), _ptr(ow), _ptr(out), _code(out), 1 if accumulate else 0,
               _ptr(ws), ws.numel(), _stream(device))
    return out


def grid_attention_prepare(pair: torch.Tensor, norm_weight: torch.Tensor | None,
                           norm_bias: torch.Tensor | None, eps: float,
                           bias_weight: torch.Tensor, num_head: int):
    """Grid attention stage 1 on pair rows: x = LN(rows) bf16 [rows, n, c] and the
    bias rows [heads, rows, n] bf16 (attention.py:86-98), in the units
    grid_attention_rows expects."""
    device = _check_cuda(pair, bias_weight)
    rows, n, c = _rows_of(pair, "pair")
    pair = _contig(pair)
    x = torch.empty((rows, n, c), dtype=torch.bfloat16, device=device)
    bias = torch.empty((num_head, rows, n), dtype=torch.bfloat16, device=device)
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    bw = prepare_weight(bias_weight)
    _capi.call("xfb_grid_attention_prepare", _ptr(pair), _code(pair), rows, n, c, num_head,
               _ptr(nw), _ptr(nb), float(eps), _ptr(bw), _ptr(x), _ptr(bias), _stream(device))
    return x, bias


def grid_attention_rows(x: torch.Tensor, mask: torch.Tensor | None, bias: torch.Tensor,
                        packed: torch.Tensor, output_weight: torch.Tensor, num_head: int,
                        out: torch.Tensor | None = None, accumulate: bool = False,
                        out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Grid attention stage 2: x = LN'd rows [rows, n, c] (pair rows, or pair
    columns for the ending node), mask [rows, n] key mask of those rows, bias
    [heads, n, n] assembled from stage 1 of every row block (attention.py:61-78,
    99-105)."""
    device = _check_cuda(x, mask, bias, packed, output_weight)
    rows, n, c = _rows_of(x, "x")
    x = _contig(x, torch.bfloat16)
    if mask is not None:
        mask = _contig(mask.expand(rows, n), torch.float32)
    bias = _contig(bias, torch.bfloat16)
    if bias.shape != (num_head, n, n):
        raise ValueError("bias must be [heads, n, n]")
    if out is None:
        if accumulate:
            raise ValueError("accumulate=True needs an output tensor")
        out = torch.empty((rows, n, c), dtype=out_dtype, device=device)
    ow = prepare_weight(output_weight)
    ws = _workspace(_capi.load().xfb_grid_attention_rows_workspace(rows, n, c, num_head), device)
    _capi.call("xfb_grid_attention_rows", _ptr(x), rows, n, c, num_head, _ptr(mask), _ptr(bias),
               _ptr(packed), _ptr(ow), _ptr(out), _code(out), 1 if accumulate else 0, _ptr(ws),
               ws.numel(), _stream(device))
    return out


def grid_attention_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        mask: torch.Tensor | None, bias: torch.Tensor,
                        gate: torch.Tensor | None, out: torch.Tensor | None = None) -> torch.Tensor:
    """The attention kernel of grid attention stage 2 alone (attention.py:61-78):
    q, k, v [rows, heads, n, 32] bf16 with q carrying log2(e)/sqrt(32), bias
    [heads, n, n] bf16 in base-2 units, mask [rows, n] key mask or None, gate
    [rows, n, heads*32] bf16 (sigmoid applied) or None; returns out [rows, n,
    heads*32] bf16."""
    device = _check_cuda(q, k, v, mask, bias, gate, out)
    rows, heads, n, d = q.shape
    if d != 32 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("the attention core takes q, k, v [rows, heads, n, 32]")
    if bias.shape != (heads, n, n):
        raise ValueError("bias must be [heads, n, n]")
    q, k, v, bias = (_contig(t, torch.bfloat16) for t in (q, k, v, bias))
    if mask is not None:
        mask = _contig(mask.expand(rows, n), torch.float32)
    if gate is not None:
        gate = _contig(gate, torch.bfloat16)
    if out is None:
        out = torch.empty((rows, n, heads * 32), dtype=torch.bfloat16, device=device)
    ws = _workspace(_capi.load().xfb_grid_attention_core_workspace(rows, n), device)
    _capi.call("xfb_grid_attention_core", _ptr(q), _ptr(k), _ptr(v), rows, heads, n, _ptr(mask),
               _ptr(bias), _ptr(gate), _ptr(out), _ptr(ws), ws.numel(), _stream(device))
    return out


def pair_logits_rows(pair: torch.Tensor, norm_weight: torch.Tensor | None,
                     norm_bias: torch.Tensor | None, eps: float,
                     weight: torch.Tensor) -> torch.Tensor:
    """Pair-logit projection of a row block: [heads, rows, n] bf16
    (pairformer.py:103-106)."""
    device = _check_cuda(pair, weight)
    rows, n, c = pair.shape
    heads = weight.shape[0]
    pair = _contig(pair)
    logits = torch.empty((heads, rows, n), dtype=torch.bfloat16, device=device)
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    w = prepare_weight(weight)
    _capi.call("xfb_pair_logits_rows", _ptr(pair), _code(pair), rows, n, c, heads, _ptr(nw),
               _ptr(nb), float(eps), _ptr(w), _ptr(logits), _stream(device))
    return logits


# ----------------------------------------------------------------------------- routed stages
# Row-block stages whose following exchange is done by the producing kernel:
# every output row is stored straight into the receive buffer of the rank that
# needs it (include/xfold_b200.h, "Routed stages").


class Route:
    """Destinations of a routed stage: dst[s] = device address of rank s's
    receive buffer as mapped in this process (dst[rank] is this GPU's own)."""

    def __init__(self, dst, rank: int) -> None:
        import ctypes

        if not 1 <= len(dst) <= 16 or not 0 <= rank < len(dst):
            raise ValueError("a route has 1..16 ranks and this rank among them")
        self.world = len(dst)
        self.rank = rank
        self._array = (ctypes.c_void_p * len(dst))(*dst)

    @property
    def ptr(self) -> int:
        import ctypes

        return ctypes.addressof(self._array)


def triangle_projection_routed(pair: torch.Tensor, mask: torch.Tensor | None,
                               left_weight: torch.Tensor, left_bias: torch.Tensor | None,
                               left_eps: float, packed: torch.Tensor, a_route: Route,
                               b_route: Route) -> torch.Tensor:
    """triangle_projection whose a and b go straight to the channel owners
    (rows -> channels); returns the local output gate g [rows, n, c]."""
    device = _check_cuda(pair, mask, left_weight, packed)
    rows, n, c = _rows_of(pair, "pair")
    pair = _contig(pair)
    if mask is not None:
        mask = _contig(mask.expand(rows, n), torch.float32)
    g = torch.empty((rows, n, c), dtype=torch.bfloat16, device=device)
    lw, lb = _contig(left_weight, torch.float32), _contig(left_bias, torch.float32)
    ws = _workspace(_capi.load().xfb_triangle_projection_workspace(rows, n, c), device)
    _capi.call("xfb_triangle_projection_routed", _ptr(pair), _code(pair), rows, n, c, _ptr(mask),
               _ptr(lw), _ptr(lb), float(left_eps), _ptr(packed), a_route.ptr, b_route.ptr,
               a_route.world, a_route.rank, _ptr(g), _ptr(ws), ws.numel(), _stream(device))
    return g


def triangle_contraction_routed(a: torch.Tensor, b: torch.Tensor, outgoing: bool,
                                z_route: Route) -> None:
    """triangle_contraction whose rows go straight to their owners (channels ->
    rows): z_route's buffers are [world * cs, n / world, n] bf16."""
    device = _check_cuda(a, b)
    a, b = _contig(a, torch.bfloat16), _contig(b, torch.bfloat16)
    cs, n, _ = a.shape
    if b.shape != a.shape:
        raise ValueError("a and b must have the same [cs, n, n] shape")
    _capi.call("xfb_triangle_contraction_routed", _ptr(a), _ptr(b), cs, n, int(bool(outgoing)),
               z_route.ptr, z_route.world, z_route.rank, _stream(device))


def grid_attention_prepare_routed(pair: torch.Tensor, norm_weight: torch.Tensor | None,
                                  norm_bias: torch.Tensor | None, eps: float,
                                  bias_weight: torch.Tensor, num_head: int,
                                  x_route: Route) -> torch.Tensor:
    """grid_attention_prepare for the ending node: the LayerNorm'd rows go
    straight to the column owners (the transpose); returns the local bias rows."""
    device = _check_cuda(pair, bias_weight)
    rows, n, c = _rows_of(pair, "pair")
    pair = _contig(pair)
    bias = torch.empty((num_head, rows, n), dtype=torch.bfloat16, device=device)
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    bw = prepare_weight(bias_weight)
    _capi.call("xfb_grid_attention_prepare_routed", _ptr(pair), _code(pair), rows, n, c, num_head,
               _ptr(nw), _ptr(nb), float(eps), _ptr(bw), x_route.ptr, x_route.world,
               x_route.rank, _ptr(bias), _stream(device))
    return bias


def grid_attention_rows_routed(x: torch.Tensor, mask: torch.Tensor | None, bias: torch.Tensor,
                               packed: torch.Tensor, output_weight: torch.Tensor, num_head: int,
                               out_route: Route) -> None:
    """grid_attention_rows for the ending node: the bf16 update goes straight
    back to the owners of the pair rows (the transpose back)."""
    device = _check_cuda(x, mask, bias, packed, output_weight)
    rows, n, c = _rows_of(x, "x")
    x = _contig(x, torch.bfloat16)
    if mask is not None:
        mask = _contig(mask.expand(rows, n), torch.float32)
    bias = _contig(bias, torch.bfloat16)
    if bias.shape != (num_head, n, n):
        raise ValueError("bias must be [heads, n, n]")
    ow = prepare_weight(output_weight)
    ws = _workspace(_capi.load().xfb_grid_attention_rows_workspace(rows, n, c, num_head), device)
    _capi.call("xfb_grid_attention_rows_routed", _ptr(x), rows, n, c, num_head, _ptr(mask),
               _ptr(bias), _ptr(packed), _ptr(ow), out_route.ptr, out_route.world,
               out_route.rank, _ptr(ws), ws.numel(), _stream(device))


def self_attention_rows(x: torch.Tensor, mask: torch.Tensor | None, logits_rows: torch.Tensor,
                        row0: int, norm_weight: torch.Tensor | None,
                        norm_bias: torch.Tensor | None, eps: float, packed: torch.Tensor,
                        q_bias: torch.Tensor | None, wo: torch.Tensor, num_head: int,
                        out: torch.Tensor, accumulate: bool = True) -> torch.Tensor:
    """The single track's attention for query rows [row0, row0 + q_rows) of x
    [n, c] (pairformer.py:102-108 for those rows) with their pair logits
    [heads, q_rows, n]; the update of those rows is written (or added) into
    `out` [n, c]."""
    device = _check_cuda(x, mask, logits_rows, packed, wo, out)
    n, c = x.shape
    q_rows = logits_rows.shape[1]
    if logits_rows.shape != (num_head, q_rows, n):
        raise ValueError("logits_rows must be [heads, q_rows, n]")
    x = _contig(x)
    if mask is not None:
        mask = _contig(mask.expand(n), torch.float32)
    logits_rows = _contig(logits_rows, torch.bfloat16)
    if not out.is_contiguous() or out.shape != (n, c):
        raise ValueError("out must be a contiguous [n, c] tensor")
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    qb, wo = _contig(q_bias, torch.float32), prepare_weight(wo)
    ws = _workspace(_capi.load().xfb_self_attention_rows_workspace(n, c, num_head, q_rows), device)
    _capi.call("xfb_self_attention_rows", _ptr(x), _code(x), n, c, num_head, row0, q_rows,
               _ptr(mask), _ptr(logits_rows), _ptr(nw), _ptr(nb), float(eps), _ptr(packed),
               _ptr(qb), _ptr(wo), None, _ptr(out), _code(out), 1 if accumulate else 0,
               _ptr(ws), ws.numel(), _stream(device))
    return out


def conditioning(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, chunk: int,
                 sig_mode: int) -> torch.Tensor:
    """act(x @ weight^T + bias) as [n / chunk, m, chunk] bf16 (one contiguous
    tensor per chunk); act = sigmoid on every chunk (sig_mode 2), on the even
    chunks (1) or none (0)."""
    device = _check_cuda(x, weight, bias)
    x, weight = _contig(x, torch.bfloat16), _contig(weight, torch.bfloat16)
    m, k = x.shape
    n = weight.shape[0]
    out = torch.empty((n // chunk, m, chunk), dtype=torch.bfloat16, device=device)
    b = _contig(bias, torch.float32)
    _capi.call("xfb_conditioning", _ptr(x), m, k, _ptr(weight), n, _ptr(b), chunk, sig_mode,
               _ptr(out), _stream(device))
    return out


# ----------------------------------------------------------------------------- atom cross-attention

def cross_pair_logits(pair_cond: torch.Tensor, norm_weight: torch.Tensor | None,
                      norm_bias: torch.Tensor | None, eps: float, weight: torch.Tensor,
                      num_blocks: int, num_head: int) -> torch.Tensor:
    """[blocks, subsets, heads, nq, nk] bf16 = rearrange(LN(pair_cond) @ weight^T,
    'n q k (b h) -> b n h q k') (xfold/nn/diffusion_transformer.py:376-380)."""
    device = _check_cuda(pair_cond, weight)
    if pair_cond.dim() != 4:
        raise ValueError("pair_cond must be [subsets, queries, keys, channels]")
    s, nq, nk, c = pair_cond.shape
    if weight.shape != (num_blocks * num_head, c):
        raise ValueError("pair logits weight must be [blocks * heads, channels]")
    pair_cond = _contig(pair_cond)
    logits = torch.empty((num_blocks, s, num_head, nq, nk), dtype=torch.bfloat16, device=device)
    nw, nb = _contig(norm_weight, torch.float32), _contig(norm_bias, torch.float32)
    w = prepare_weight(weight)
    _capi.call("xfb_cross_pair_logits", _ptr(pair_cond), _code(pair_cond), s, nq, nk, c,
               num_blocks, num_head, _ptr(nw), _ptr(nb), float(eps), _ptr(w), _ptr(logits),
               _stream(device))
    return logits


def pack_cross_attention_weights(q_w: torch.Tensor, gate_w: torch.Tensor, k_w: torch.Tensor,
                                 v_w: torch.Tensor) -> torch.Tensor:
    """[4c, c] bf16 rows q_projection | gating_query | k_projection | v_projection."""
    return pack_attention_weights(q_w, gate_w, k_w, v_w)


def cross_attention(x_q: torch.Tensor, keys, mask_q: torch.Tensor | None,
                    mask_k: torch.Tensor | None, pair_logits: torch.Tensor | None, eps: float,
                    packed: torch.Tensor, q_bias: torch.Tensor | None, wo: torch.Tensor,
                    q_mod: tuple | None = None, k_mod: tuple | None = None,
                    out_gate: torch.Tensor | None = None, out: torch.Tensor | None = None,
                    accumulate: bool = False,
                    out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """CrossAttention update (xfold/nn/diffusion_transformer.py:307-350) over
    windows of 32 queries x 128 keys, c = 128, 4 heads.

    x_q [subsets, 32, 128]; keys is either x_k [subsets, 128, 128] or a pair
    (index [subsets, 128] int64, valid [subsets, 128] bool) selecting rows of
    x_q flattened to [subsets*32, 128] (valid False -> zero row), the
    queries_to_keys gather fused into the keys' LayerNorm.  q_mod / k_mod are
    (sigmoid(scale), shift) of the adaptive LayerNorms, out_gate the AdaLNZero
    gate, all [rows, 128] bf16."""
    device = _check_cuda(x_q, packed, wo, pair_logits, out_gate)
    if x_q.dim() != 3:
        raise ValueError("x_q must be [subsets, queries, channels]")
    s, nq, c = x_q.shape
    nk = 128
    x_q = _contig(x_q)
    x_k = index = valid = None
    rows = s * nq
    if isinstance(keys, torch.Tensor):
        _check_cuda(keys)
        if keys.dim() != 3 or keys.shape[0] != s or keys.shape[2] != c:
            raise ValueError("x_k must be [subsets, keys, channels]")
        nk = keys.shape[1]
        x_k = _contig(keys, x_q.dtype)
    else:
        index, valid = keys
        _check_cuda(index, valid)
        if index.shape != valid.shape or index.dim() != 2 or index.shape[0] != s:
            raise ValueError("key gather index and mask must both be [subsets, keys]")
        nk = index.shape[1]
        index = _contig(index, torch.int64)
        valid = _contig(valid, torch.bool)
    if mask_q is not None:
        mask_q = _contig(mask_q.expand(s, nq), torch.float32)
    if mask_k is not None:
        mask_k = _contig(mask_k.expand(s, nk), torch.float32)
    if pair_logits is not None:
        if tuple(pair_logits.shape[-3:]) != (4, nq, nk):
            raise ValueError("pair logits must be [subsets, heads, queries, keys]")
        pair_logits = _contig(pair_logits, torch.bfloat16)
    qs, qh = (None, None) if q_mod is None else (_contig(t, torch.bfloat16) for t in q_mod)
    ks, kh = (None, None) if k_mod is None else (_contig(t, torch.bfloat16) for t in k_mod)
    out_gate = _contig(out_gate, torch.bfloat16)
    if out is None:
        out = torch.empty((s, nq, c), dtype=out_dtype, device=device)
    qb, wo = _contig(q_bias, torch.float32), prepare_weight(wo)
    ws = _workspace(_capi.load().xfb_cross_attention_workspace(s), device)
    _capi.call("xfb_cross_attention", _ptr(x_q), _code(x_q), s, nq, nk, c, 4, _ptr(x_k),
               _ptr(index), _ptr(valid), rows, _ptr(mask_q), _ptr(mask_k), _ptr(pair_logits),
               float(eps), _ptr(qs), _ptr(qh), _ptr(ks), _ptr(kh), _ptr(packed), _ptr(qb),
               _ptr(wo), _ptr(out_gate), _ptr(out), _code(out), 1 if accumulate else 0, _ptr(ws),
               ws.numel(), _stream(device))
    return out


# ----------------------------------------------------------------------------- MSA stack

def msa_attention(msa: torch.Tensor, msa_mask: torch.Tensor | None, pair: torch.Tensor,
                  act_norm_w: torch.Tensor | None, act_norm_b: torch.Tensor | None,
                  pair_norm_w: torch.Tensor | None, pair_norm_b: torch.Tensor | None, eps: float,
                  pair_logits_w: torch.Tensor, v_w: torch.Tensor, gate_w: torch.Tensor,
                  out_w: torch.Tensor, out: torch.Tensor | None = None, accumulate: bool = False,
                  out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """MSAAttention update (xfold/nn/attention.py:125-144): msa [S, N, 64],
    msa_mask [S, N], pair [N, N, 128]; 8 heads of 8."""
    device = _check_cuda(msa, pair, msa_mask, pair_logits_w, v_w, gate_w, out_w)
    if msa.dim() != 3 or pair.dim() != 3:
        raise ValueError("msa must be [S, N, c_msa] and pair [N, N, c_pair]")
    s, n, c = msa.shape
    msa, pair = _contig(msa), _contig(pair)
    if msa_mask is not None:
        msa_mask = _contig(msa_mask.expand(s, n), torch.float32)
    if out is None:
        out = torch.empty((s, n, c), dtype=out_dtype, device=device)
    f32 = [_contig(t, torch.float32) for t in (act_norm_w, act_norm_b, pair_norm_w, pair_norm_b)]
    ws_w = [prepare_weight(t) for t in (pair_logits_w, v_w, gate_w, out_w)]
    ws = _workspace(_capi.load().xfb_msa_attention_workspace(s, n), device)
    _capi.call("xfb_msa_attention", _ptr(msa), _code(msa), s, n, c, _ptr(msa_mask), _ptr(pair),
               _code(pair), pair.shape[-1], pair_logits_w.shape[0], *(_ptr(t) for t in f32),
               float(eps), *(_ptr(t) for t in ws_w), _ptr(out), _code(out),
               1 if accumulate else 0, _ptr(ws), ws.numel(), _stream(device))
    return out


def pack_outer_product_weight(output_w: torch.Tensor) -> torch.Tensor:
    """output_w [32, 32, f] -> [f, 1024] bf16 (the second contraction's operand)."""
    device = _check_cuda(output_w)
    if output_w.dim() != 3 or output_w.shape[:2] != (32, 32):
        raise ValueError("output_w must be [32, 32, f]")
    w = _contig(output_w)
    f = w.shape[2]
    packed = torch.empty((f, 1024), dtype=torch.bfloat16, device=device)
    _capi.call("xfb_pack_outer_product_weight", _ptr(w), _code(w), f, _ptr(packed), _stream(device))
    return packed


def outer_product_mean(msa: torch.Tensor, mask: torch.Tensor, norm_w: torch.Tensor | None,
                       norm_b: torch.Tensor | None, eps: float, left_w: torch.Tensor,
                       right_w: torch.Tensor, packed_output_w: torch.Tensor,
                       output_b: torch.Tensor, out: torch.Tensor | None = None,
                       accumulate: bool = False) -> torch.Tensor:
    """OuterProductMean update (xfold/nn/primitives.py:62-75): msa [S, N, 64],
    mask [S, N] -> [N, N, 128] f32."""
    device = _check_cuda(msa, mask, left_w, right_w, packed_output_w, output_b)
    if msa.dim() != 3:
        raise ValueError("msa must be [S, N, c_msa]")
    s, n, c = msa.shape
    msa = _contig(msa)
    mask = _contig(mask.expand(s, n), torch.float32)
    c_out = packed_output_w.shape[0]
    if out is None:
        out = torch.empty((n, n, c_out), dtype=torch.float32, device=device)
    elif out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("outer product mean writes a contiguous f32 [N, N, c] tensor")
    nw, nb, ob = (_contig(t, torch.float32) for t in (norm_w, norm_b, output_b))
    lw, rw = prepare_weight(left_w), prepare_weight(right_w)
    ws = _workspace(_capi.load().xfb_outer_product_mean_workspace(s, n), device)
    _capi.call("xfb_outer_product_mean", _ptr(msa), _code(msa), s, n, c, _ptr(mask), _ptr(nw),
               _ptr(nb), float(eps), _ptr(lw), _ptr(rw), _ptr(packed_output_w), _ptr(ob), c_out,
               _ptr(out), 1 if accumulate else 0, _ptr(ws), ws.numel(), _stream(device))
    return out
