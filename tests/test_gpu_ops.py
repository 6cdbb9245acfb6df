"""Operator parity on the GPU: every C-ABI operator against the CPU oracle.

Tolerance: max|got - ref| / max|ref| <= 1e-2 for the bf16 CUDA path against
the float32 oracle (the bf16 bar of the north star), measured on the update.
"""

import pytest
import torch

import oracle
from xfold_cpu_b200 import native

pytestmark = pytest.mark.gpu

TOL = 1e-2
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_error():
    """Every operator must finish without a bounded wait expiring."""
    from xfold_cpu_b200 import _capi

    _capi.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert _capi.device_error(clear=True) == 0


def _g(seed):
    return torch.Generator().manual_seed(seed)


def _w(g, *shape, std=0.02):
    return torch.randn(*shape, generator=g) * std


def _ln(g, c):
    return 1.0 + 0.1 * torch.randn(c, generator=g), 0.1 * torch.randn(c, generator=g)


def _rel(got, ref):
    return oracle.relative_error(got.float().cpu(), ref)


@pytest.mark.parametrize("m,k,n", [(256, 128, 512), (1000, 128, 640), (77, 384, 136), (300, 512, 128)])
def test_linear(m, k, n):
    g = _g(1)
    x = torch.randn(m, k, generator=g)
    w = _w(g, n, k, std=0.05)
    b = torch.randn(n, generator=g)
    ref = oracle.linear(x.bfloat16().float(), w.bfloat16().float(), b)
    got = native.linear(x.to(DEV), w.to(DEV), b.to(DEV), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _rel(got, ref) < 5e-3


@pytest.mark.parametrize("rows,c", [(1000, 128), (33, 64), (257, 384), (64, 768)])
def test_layer_norm(rows, c):
    g = _g(2)
    x = torch.randn(rows, c, generator=g) * 3 + 1
    w, b = _ln(g, c)
    ref = oracle.layer_norm(x, w, b)
    got = native.layer_norm(x.to(DEV), w.to(DEV), b.to(DEV))
    assert _rel(got, ref) < 8e-3


@pytest.mark.parametrize("rows,dtype", [(1001, torch.float32), (6, torch.float32),
                                        (4099, torch.bfloat16)])
def test_layer_norm_multirow_tails(rows, dtype):
    """The 128-wide LayerNorm takes four rows per warp: row counts that leave a
    partial group, fewer rows than one group's warps, and bf16 input."""
    g = _g(12)
    x = (torch.randn(rows, 128, generator=g) * 2 - 0.5).to(dtype)
    w, b = _ln(g, 128)
    ref = oracle.layer_norm(x.float(), w, b)
    got = native.layer_norm(x.to(DEV), w.to(DEV), b.to(DEV))
    assert _rel(got, ref) < 8e-3


@pytest.mark.parametrize("m,k,n", [(500, 128, 512), (129, 384, 1536)])
def test_gated_linear_unit(m, k, n):
    g = _g(3)
    x = torch.randn(m, k, generator=g)
    w = _w(g, 2 * n, k, std=0.1)
    ref = oracle.gated_linear_unit(x.bfloat16().float(), w.bfloat16().float().T)
    got = native.gated_linear_unit(x.to(DEV).bfloat16(), w.to(DEV))
    assert _rel(got, ref) < TOL


def _attention_case(B, H, nq, nk, d, mask_kind, bias_kind, seed=4):
    g = _g(seed)
    q = torch.randn(B, H, nq, d, generator=g)
    k = torch.randn(B, H, nk, d, generator=g)
    v = torch.randn(B, H, nk, d, generator=g)
    mask = None
    if mask_kind == "rank1":
        mask = (torch.rand(nk, generator=g) > 0.3).float()
    elif mask_kind == "rank2":
        mask = (torch.rand(B, nk, generator=g) > 0.3).float()
        mask[0] = 0  # a fully masked row: uniform softmax
    elif mask_kind == "tail":
        mask = torch.ones(nk)
        mask[-min(64, nk // 2):] = 0
    bias = None
    if bias_kind == "shared":
        bias = torch.randn(H, nq, nk, generator=g)
    elif bias_kind == "batched":
        bias = torch.randn(B, H, nq, nk, generator=g)
    return q, k, v, mask, bias


@pytest.mark.parametrize("B,H,nq,nk,d,mask_kind,bias_kind", [
    (2, 4, 256, 256, 32, "rank2", "shared"),
    (3, 4, 200, 200, 32, "rank1", "batched"),
    (1, 16, 300, 300, 24, "tail", "shared"),
    (2, 2, 130, 130, 48, None, "batched"),
    (1, 2, 64, 1000, 64, "rank1", None),
    (2, 4, 128, 128, 16, "rank2", "shared"),
])
def test_dot_product_attention(B, H, nq, nk, d, mask_kind, bias_kind):
    q, k, v, mask, bias = _attention_case(B, H, nq, nk, d, mask_kind, bias_kind)
    rb = lambda t: None if t is None else t.bfloat16().float()
    ref = oracle.dot_product_attention(rb(q), rb(k), rb(v), mask, rb(bias))
    dev = lambda t: None if t is None else t.to(DEV)
    got = native.dot_product_attention(dev(q), dev(k), dev(v), dev(mask),
                                       None if bias is None else bias.to(DEV).bfloat16())
    assert _rel(got, ref) < TOL


@pytest.mark.parametrize("B,H,n,d", [(50, 4, 200, 32), (49, 8, 136, 16), (48, 4, 64, 32)])
def test_dot_product_attention_three_slot_kernel(B, H, n, d):
    """Shapes with >= 48 batch rows and one shared bias run on the three-slot
    kernel: a batch not divisible by 3, ragged query / key tiles, a fully
    masked row and tail-masked rows.  Checked against the oracle and against
    the one-tile kernel (the same rows two at a time)."""
    g = _g(9)
    q = torch.randn(B, H, n, d, generator=g) * 0.5
    k = torch.randn(B, H, n, d, generator=g) * 0.5
    v = torch.randn(B, H, n, d, generator=g)
    bias = torch.randn(H, n, n, generator=g)
    mask = torch.ones(B, n)
    mask[:, -max(1, n // 10):] = 0
    mask[3] = 0  # every key of row 3 masked: a uniform average
    mask[7, : n // 2] = 0
    rb = lambda t: t.bfloat16().float()
    ref = oracle.dot_product_attention(rb(q), rb(k), rb(v), mask, rb(bias)[None])
    dq, dk, dv, dm = q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV)
    db = bias.to(DEV).bfloat16()
    got = native.dot_product_attention(dq, dk, dv, dm, db)
    assert _rel(got, ref) < TOL
    one_tile = torch.cat([native.dot_product_attention(dq[i:i + 2], dk[i:i + 2], dv[i:i + 2],
                                                       dm[i:i + 2], db)
                          for i in range(0, B, 2)])
    assert _rel(got, one_tile.float().cpu()) < 8e-3  # two bf16 ulps of the largest output


def _tri_params(g, c):
    lw, lb = _ln(g, c)
    cw, cb = _ln(g, c)
    return {
        "left_norm_input.weight": lw, "left_norm_input.bias": lb,
        "projection.weight": _w(g, 2 * c, c), "gate.weight": _w(g, 2 * c, c),
        "center_norm.weight": cw, "center_norm.bias": cb,
        "output_projection.weight": _w(g, c, c), "gating_linear.weight": _w(g, c, c),
    }


@pytest.mark.parametrize("n,c,outgoing", [(64, 128, True), (64, 128, False), (130, 128, True),
                                          (130, 128, False), (200, 64, False), (256, 128, True)])
def test_triangle_multiplication(n, c, outgoing):
    g = _g(5)
    p = _tri_params(g, c)
    pair = torch.randn(n, n, c, generator=g)
    m = torch.ones(n)
    m[-max(1, n // 20):] = 0
    mask = m[:, None] * m[None, :]
    ref = oracle.triangle_multiplication(pair, mask, p, outgoing)
    d = {k: v.to(DEV) for k, v in p.items()}
    got = native.triangle_multiplication(
        pair.to(DEV), mask.to(DEV), outgoing, d["left_norm_input.weight"], d["left_norm_input.bias"],
        d["projection.weight"], d["gate.weight"], d["center_norm.weight"], d["center_norm.bias"],
        d["output_projection.weight"], d["gating_linear.weight"], out_dtype=torch.float32)
    assert _rel(got, ref) < TOL


def _gsa_params(g, c, heads):
    w, b = _ln(g, c)
    return {
        "act_norm.weight": w, "act_norm.bias": b,
        "pair_bias_projection.weight": _w(g, heads, c, std=0.1),
        "q_projection.weight": _w(g, c, c, std=0.1), "k_projection.weight": _w(g, c, c, std=0.1),
        "v_projection.weight": _w(g, c, c), "gating_query.weight": _w(g, c, c),
        "output_projection.weight": _w(g, c, c),
    }


@pytest.mark.parametrize("n,c,heads,transpose", [(64, 128, 4, False), (64, 128, 4, True),
                                                 (150, 128, 4, True), (96, 64, 4, False)])
def test_grid_self_attention(n, c, heads, transpose):
    g = _g(6)
    p = _gsa_params(g, c, heads)
    pair = torch.randn(n, n, c, generator=g)
    m = torch.ones(n)
    m[-max(1, n // 10):] = 0
    mask = m[:, None] * m[None, :]
    ref = oracle.grid_self_attention(pair, mask, p, transpose, heads)
    d = {k: v.to(DEV) for k, v in p.items()}
    packed = native.pack_attention_weights(d["q_projection.weight"], d["k_projection.weight"],
                                           d["v_projection.weight"], d["gating_query.weight"])
    got = native.grid_self_attention(pair.to(DEV), mask.to(DEV), transpose, d["act_norm.weight"],
                                     d["act_norm.bias"], 1e-5, d["pair_bias_projection.weight"],
                                     packed, d["output_projection.weight"], heads,
                                     out_dtype=torch.float32)
    assert _rel(got, ref) < TOL


@pytest.mark.parametrize("rows,c,factor", [(4096, 128, 4), (300, 384, 4), (200, 768, 2)])
def test_transition(rows, c, factor):
    g = _g(7)
    w, b = _ln(g, c)
    p = {"input_layer_norm.weight": w, "input_layer_norm.bias": b,
         "transition1.weight": _w(g, 2 * factor * c, c, std=0.1),
         "transition2.weight": _w(g, c, factor * c, std=0.05)}
    x = torch.randn(rows, c, generator=g)
    ref = oracle.transition(x, p)
    d = {k: v.to(DEV) for k, v in p.items()}
    w1 = native.pack_glu_weight(d["transition1.weight"])
    got = native.transition(x.to(DEV), d["input_layer_norm.weight"], d["input_layer_norm.bias"],
                            1e-5, w1, d["transition2.weight"], factor, out_dtype=torch.float32)
    assert _rel(got, ref) < TOL


@pytest.mark.parametrize("rows,factor,accumulate", [(300, 4, True), (1000, 2, False),
                                                     (128, 4, False)])
def test_fused_pair_transition(rows, factor, accumulate):
    """c = 128 with an f32 output runs the fused GLU transition (hidden tile kept
    on chip): a partial last row tile, hidden 256 / 512, residual add and store."""
    g = _g(8)
    c = 128
    w, b = _ln(g, c)
    p = {"input_layer_norm.weight": w, "input_layer_norm.bias": b,
         "transition1.weight": _w(g, 2 * factor * c, c, std=0.1),
         "transition2.weight": _w(g, c, factor * c, std=0.05)}
    x = torch.randn(rows, c, generator=g)
    base = torch.randn(rows, c, generator=g)
    ref = oracle.transition(x, p)
    d = {k: v.to(DEV) for k, v in p.items()}
    w1 = native.pack_glu_weight(d["transition1.weight"])
    out = base.to(DEV).clone() if accumulate else None
    got = native.transition(x.to(DEV), d["input_layer_norm.weight"], d["input_layer_norm.bias"],
                            1e-5, w1, d["transition2.weight"], factor, out=out,
                            accumulate=accumulate, out_dtype=torch.float32)
    update = got.cpu() - base if accumulate else got.cpu()
    assert _rel(update, ref) < TOL


@pytest.mark.parametrize("n,c,heads", [(200, 384, 16), (300, 768, 16)])
def test_self_attention(n, c, heads):
    g = _g(8)
    w, b = _ln(g, c)
    p = {"adaptive_layernorm.layer_norm.weight": w, "adaptive_layernorm.layer_norm.bias": b,
         "q_projection.weight": _w(g, c, c, std=0.05), "q_projection.bias": 0.1 * torch.randn(c, generator=g),
         "k_projection.weight": _w(g, c, c, std=0.05), "v_projection.weight": _w(g, c, c),
         "gating_query.weight": _w(g, c, c), "adaptive_zero_init.transition2.weight": _w(g, c, c)}
    x = torch.randn(n, c, generator=g)
    mask = torch.ones(n)
    mask[-7:] = 0
    logits = torch.randn(heads, n, n, generator=g)
    ref = oracle.self_attention(x, mask, logits.bfloat16().float(), p, None, heads, False)
    d = {k: v.to(DEV) for k, v in p.items()}
    packed = native.pack_attention_weights(d["q_projection.weight"], d["k_projection.weight"],
                                           d["v_projection.weight"], d["gating_query.weight"])
    got = native.self_attention(x.to(DEV), mask.to(DEV), logits.to(DEV), d["adaptive_layernorm.layer_norm.weight"],
                                d["adaptive_layernorm.layer_norm.bias"], 1e-5, packed,
                                d["q_projection.bias"], d["adaptive_zero_init.transition2.weight"], heads,
                                out_dtype=torch.float32)
    assert _rel(got, ref) < TOL


def test_pair_logits():
    g = _g(9)
    n, c, h = 100, 128, 16
    w, b = _ln(g, c)
    p = {"single_pair_logits_norm.weight": w, "single_pair_logits_norm.bias": b,
         "single_pair_logits_projection.weight": _w(g, h, c, std=0.2)}
    pair = torch.randn(n, n, c, generator=g)
    ref = oracle.pair_logits(pair, p)
    d = {k: v.to(DEV) for k, v in p.items()}
    got = native.pair_logits(pair.to(DEV), d["single_pair_logits_norm.weight"],
                             d["single_pair_logits_norm.bias"], 1e-5,
                             d["single_pair_logits_projection.weight"])
    assert _rel(got, ref) < TOL


def test_bounded_wait_reports_timeout():
    """A device wait that nothing satisfies gives up and reports a status."""
    from xfold_cpu_b200 import _capi

    _capi.call("xfb_selftest_wait_timeout", 50_000_000, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _capi.device_error(clear=True) == 0x1FF
    # the context is still usable afterwards
    x = torch.ones(4, device=DEV)
    assert float(x.sum()) == 4.0


@pytest.mark.parametrize("m,k,chunks,chunk,sig_mode", [
    (200, 128, 6, 128, 1),   # atom rows: AdaLN (scale, shift) pairs
    (768, 384, 4, 768, 2),   # token rows: AdaLNZero gates
    (37, 128, 3, 128, 0),
])
def test_conditioning(m, k, chunks, chunk, sig_mode):
    """act(x W^T + b) in the chunked [n / chunk, m, chunk] layout."""
    g = _g(50 + sig_mode)
    n = chunks * chunk
    x = torch.randn(m, k, generator=g).bfloat16()
    w = _w(g, n, k, std=0.1).bfloat16()
    b = torch.randn(n, generator=g)
    ref = (x.float() @ w.float().T + b).reshape(m, chunks, chunk).permute(1, 0, 2)
    sig = torch.tensor([sig_mode == 2 or (sig_mode == 1 and q % 2 == 0) for q in range(chunks)])
    ref = torch.where(sig[:, None, None], torch.sigmoid(ref), ref)
    got = native.conditioning(x.to(DEV), w.to(DEV), b.to(DEV), chunk, sig_mode)
    assert got.shape == (chunks, m, chunk)
    assert oracle.relative_error(got.float().cpu(), ref) < TOL
