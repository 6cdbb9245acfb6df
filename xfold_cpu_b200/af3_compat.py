"""The reference's native extension API (af3_kernels) on CUDA tensors.

xfold's CPU backend calls `af3_kernels._C` through `load_native_operator(name)`
(xfold/fastnn/native.py:7-18) with the argument lists of
af3_kernels/src/csrc/bindings.cpp:26-49.  This module exposes the same
functions, arguments and defaults for CUDA tensors, backed by the
`xfb_af3_*` entry points of libxfold_b200.so, so xfold's own bridges
(`TriangleMultiplication._forward_cpp`, `linear_cpp`,
`dot_product_attention_cpp`) can drive the B200 kernels unchanged once their
CPU-only device checks accept CUDA tensors (INTEGRATION.md shows the patch).

Weights are the transposed nn.Linear weights `[in, out]` the bridges pass.
The CPU tile sizes (`block_size`, `M_BLK`, `N_BLK`, `query_block`) are
checked like the reference's `xsmm_size` and do not change results.  The
VNNI2 packed-weight layout is a CPU format: `weights_packed=True` raises, and
`packed_weight_api` is 0, so xfold's packed-weight cache is not used with this
module.  Results come back in the input dtype; the arithmetic is bf16 with f32
accumulation (the reference's GPU route is bf16 autocast).
"""

from __future__ import annotations

import math

import torch

from . import _capi, native

packed_weight_api = 0


def load_extension():
    """This module plays the role of af3_kernels._C.  Like the reference's
    load_native_operator (xfold/fastnn/native.py:7-18) it raises RuntimeError
    when the native library is missing or lacks a symbol."""
    import sys

    _capi.load()
    return sys.modules[__name__]


def runtime_info() -> dict:
    return native.runtime_info()


def _check_tensor(t: torch.Tensor, what: str = "Native tools") -> None:
    """af3_detail::check_tensor (af3_kernels/src/csrc/tools.cpp:20-28) for CUDA tensors."""
    if not t.is_cuda:
        raise RuntimeError(f"{what} require CUDA tensors.")
    if t.layout != torch.strided:
        raise RuntimeError(f"{what} require strided tensors.")
    if t.dtype not in (torch.float32, torch.bfloat16):
        raise RuntimeError(f"{what} support FP32 and BF16 tensors only.")
    if t.requires_grad and torch.is_grad_enabled():
        raise RuntimeError(f"{what} support inference only.")
    if t.is_conj() or t.is_neg():
        raise RuntimeError("Resolve conjugate/negative tensor views before using native tools.")


def _block(size: int, name: str) -> None:
    if not (0 < int(size) <= 2 ** 31 - 1):
        raise RuntimeError("Matrix dimensions must fit positive LIBXSMM integers.")


def _no_vnni(packed: bool) -> None:
    if packed:
        raise RuntimeError("VNNI2-packed weights are a CPU layout; pass the [in, out] weights.")


def _wcode(t: torch.Tensor) -> int:
    return _capi.F32 if t.dtype == torch.float32 else _capi.BF16


def gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """xsmm_gemm (tools.cpp:120-150): [M, K] @ [K, N] -> float32 [M, N]."""
    _check_tensor(a)
    _check_tensor(b)
    if a.dim() != 2 or b.dim() != 2:
        raise RuntimeError("GEMM requires 2D tensors.")
    if a.dtype != b.dtype:
        raise RuntimeError("GEMM input dtypes must match.")
    if a.size(1) != b.size(0):
        raise RuntimeError("GEMM inner dimensions must match.")
    if not (a.is_contiguous() and b.is_contiguous()):
        raise RuntimeError("GEMM inputs must be contiguous.")
    m, k = a.shape
    n = b.size(1)
    out = torch.empty((m, n), dtype=torch.float32, device=a.device)
    ab, bb = a.to(torch.bfloat16).contiguous(), b.to(torch.bfloat16).contiguous()
    _capi.call("xfb_gemm", native._ptr(ab), native._ptr(bb), native._ptr(out), 1, m, n, k, 0, 1,
               _capi.F32, native._stream(a.device))
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           weight_packed: bool = False) -> torch.Tensor:
    """xsmm_linear (matrix.cpp:119-129): x [..., K] @ weight [K, N] (+ bias), in x's dtype."""
    _no_vnni(weight_packed)
    _check_tensor(x)
    if x.dim() < 1 or not x.is_contiguous():
        raise RuntimeError("Linear input must be contiguous [..., K].")
    if weight.dim() != 2:
        raise RuntimeError("Linear weight must be [K, N] or its padded packed layout.")
    _check_tensor(weight)
    k = x.size(-1)
    _block(k, "K")
    if weight.size(0) != k:
        raise RuntimeError("Linear inner dimensions must match.")
    n = weight.size(1)
    m = x.numel() // k
    xb = x.reshape(m, k).to(torch.bfloat16).contiguous()
    w = weight.contiguous()
    b = None if bias is None else bias.to(torch.float32).contiguous()
    # the kernel writes rows of a multiple of 8 outputs: narrower weights (the
    # 4-head pair-bias projection) get zero columns and an f32 buffer
    n_pad = -(-n // 8) * 8
    if n_pad != n:
        w = torch.nn.functional.pad(w, (0, n_pad - n)).contiguous()
        if b is not None:
            b = torch.nn.functional.pad(b, (0, n_pad - n)).contiguous()
    y = torch.empty((m, n_pad), dtype=x.dtype if n_pad == n else torch.float32, device=x.device)
    if m > 0:
        lib = _capi.load()
        ws = native._workspace(lib.xfb_af3_linear_workspace(k, n_pad), x.device)
        _capi.call("xfb_af3_linear", native._ptr(xb), m, k, native._ptr(w), _wcode(w), n_pad,
                   native._ptr(b), 0, native._ptr(y), native._code(y), native._ptr(ws),
                   ws.numel(), native._stream(x.device))
    if n_pad != n:
        y = y[:, :n].to(x.dtype)
    return y.reshape(*x.shape[:-1], n)


def gated_linear_unit(x: torch.Tensor, weight: torch.Tensor, M_BLK: int = 128, N_BLK: int = 128,
                      weight_packed: bool = False) -> torch.Tensor:
    """xsmm_gated_linear_unit (gated_linear_unit.cpp:78-121): silu(x W[:, :N]) * (x W[:, N:])
    for x [..., K], weight [K, 2N]; returns [..., N] in x's dtype."""
    _no_vnni(weight_packed)
    _check_tensor(x)
    _check_tensor(weight)
    if x.dim() < 1 or weight.dim() != 2:
        raise RuntimeError("GLU expects [..., K] and [K, 2*N].")
    if not (x.is_contiguous() and weight.is_contiguous()):
        raise RuntimeError("GLU inputs must be contiguous.")
    if x.dtype != weight.dtype:
        raise RuntimeError("GLU input dtypes must match.")
    k = x.size(-1)
    _block(k, "K")
    if weight.size(0) != k:
        raise RuntimeError("GLU inner dimensions must match the normal/padded packed weight.")
    width = weight.size(1)
    _block(width, "2N")
    if width % 2:
        raise RuntimeError("GLU weight width must be positive and even.")
    _block(M_BLK, "M_BLK")
    _block(N_BLK, "N_BLK")
    n = width // 2
    m = x.numel() // k
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    if m > 0:
        xb = x.reshape(m, k).to(torch.bfloat16).contiguous()
        lib = _capi.load()
        ws = native._workspace(lib.xfb_af3_gated_linear_unit_workspace(k, n), x.device)
        _capi.call("xfb_af3_gated_linear_unit", native._ptr(xb), m, k, native._ptr(weight),
                   _wcode(weight), n, int(M_BLK), int(N_BLK), 0, native._ptr(out),
                   native._ptr(ws), ws.numel(), native._stream(x.device))
    return out.to(x.dtype).reshape(*x.shape[:-1], n)


def triangle_multiplication(pair, mask, outgoing, left_weight, left_bias, projection, gate,
                            center_weight, center_bias, output_weight, gating_weight,
                            left_eps=1e-5, center_eps=1e-5, block_size=128,
                            weights_packed=False):
    """xsmm_triangle_multiplication (triangle_multiplication.cpp:6-73): the update of
    pair [N, N, C] with weights [C, 2C] / [C, C]; returns [N, N, C] in the weights' dtype."""
    _no_vnni(weights_packed)
    _check_tensor(pair)
    if pair.dim() != 3 or pair.size(0) != pair.size(1) or not pair.is_contiguous():
        raise RuntimeError("Triangle input must be contiguous [N, N, C].")
    n, c = pair.size(0), pair.size(2)
    _block(c, "C")
    _block(block_size, "block_size")
    if not all(math.isfinite(e) and e >= 0 for e in (left_eps, center_eps)):
        raise RuntimeError("LayerNorm eps must be finite and nonnegative.")
    for w in (projection, gate, output_weight, gating_weight):
        _check_tensor(w)
        if w.dim() != 2 or w.size(0) != c or not w.is_contiguous() or w.dtype != projection.dtype:
            raise RuntimeError("Invalid Triangle projection weight.")
    if projection.size(1) != 2 * c or gate.size(1) != 2 * c or output_weight.size(1) != c or \
            gating_weight.size(1) != c:
        raise RuntimeError("Triangle weight widths do not match C.")
    for w in (left_weight, center_weight):
        _check_tensor(w)
        if w.dim() != 1 or w.size(0) != c:
            raise RuntimeError("LayerNorm weights must be [C].")
    for b in (left_bias, center_bias):
        if b is not None:
            _check_tensor(b)
            if b.dim() != 1 or b.size(0) != c:
                raise RuntimeError("LayerNorm biases must be [C].")
    m = None
    if mask is not None:
        if mask.dim() > 2 or mask.is_complex():
            raise RuntimeError("Triangle mask must broadcast to [N, N].")
        m = mask.expand(n, n).to(torch.float32).contiguous()
    out = torch.empty((n, n, c), dtype=projection.dtype, device=pair.device)
    if n == 0:
        return out
    f32 = lambda t: None if t is None else t.to(torch.float32).contiguous()
    lib = _capi.load()
    ws = native._workspace(lib.xfb_af3_triangle_multiplication_workspace(n, c), pair.device)
    _capi.call("xfb_af3_triangle_multiplication", native._ptr(pair), native._code(pair), n, c,
               native._ptr(m), 1 if outgoing else 0, native._ptr(f32(left_weight)),
               native._ptr(f32(left_bias)), native._ptr(projection), native._ptr(gate),
               native._ptr(f32(center_weight)), native._ptr(f32(center_bias)),
               native._ptr(output_weight), native._ptr(gating_weight), _wcode(projection),
               float(left_eps), float(center_eps), int(block_size), 0, native._ptr(out),
               native._code(out), native._ptr(ws), ws.numel(), native._stream(pair.device))
    return out


def dot_product_attention(q, k, v, mask=None, bias=None, query_block=128, q_pre_scaled=False):
    """xsmm_dot_product_attention (dot_product_attention.cpp:110-174): q [B, H, Q, D],
    k [B, H, K, D], v [B, H, K, Dv]; mask rank 1 / 2 (any dtype) or a bool mask broadcast
    over heads and queries; bias broadcastable to [B, H, Q, K]; -1e9 for masked
    logits.  Returns [B, H, Q, Dv] in q's dtype."""
    for t in (q, k, v):
        _check_tensor(t)
        if t.dim() != 4 or not t.is_contiguous():
            raise RuntimeError("Attention requires contiguous [B, H, Q/K, D].")
        if t.dtype != q.dtype:
            raise RuntimeError("Attention Q/K/V dtypes must match.")
    if q.shape[:2] != k.shape[:2] or q.shape[:2] != v.shape[:2]:
        raise RuntimeError("Attention batch/head dimensions must match.")
    if q.size(3) != k.size(3) or k.size(2) != v.size(2):
        raise RuntimeError("Attention key/head dimensions must match.")
    _block(q.size(3), "D")
    _block(query_block, "query_block")
    if mask is not None and (mask.dim() > 4 or mask.is_complex()):
        raise RuntimeError("Invalid attention mask rank/type.")
    if bias is not None:
        _check_tensor(bias)
        if bias.dim() > 4:
            raise RuntimeError("Attention bias must broadcast to [B, H, Q, K].")
    out = native.dot_product_attention(q, k, v, mask, bias, q_pre_scaled=bool(q_pre_scaled),
                                       query_block=int(query_block))
    return out.to(q.dtype)
