"""The float32 compute path (fastnn.config.compute_dtype = "float32") against the
float32 oracle at the north_star's fp32 tolerance, 1e-4 (max |err| / max |ref|).

The oracle restates the reference's torch path in fp32 (oracle/hotpath.py,
pinned to the reference by tests/test_oracle_golden.py); the modules run the
library's CUDA-core fp32 kernels (xfb_f32_*) through xfold_cpu_b200/fp32.py."""

import pytest
import torch

import oracle
from xfold_cpu_b200 import _capi, fp32
from xfold_cpu_b200.fastnn import config
from xfold_cpu_b200.nn import (DiffusionTransformer, DiffusionTransition, GridSelfAttention,
                               PairformerBlock, SelfAttention, Transition, TriangleMultiplication,
                               init_params_)

pytestmark = pytest.mark.gpu

TOL = 1e-4
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _fp32_mode():
    _capi.device_error(clear=True)
    old = config.compute_dtype
    config.compute_dtype = config.FLOAT32
    yield
    config.compute_dtype = old
    torch.cuda.synchronize()
    assert _capi.device_error(clear=True) == 0


def _params(module):
    return {k: v.detach().cpu().clone() for k, v in module.state_dict().items()}


def _masks(n, tail):
    seq = torch.ones(n)
    seq[-tail:] = 0
    return seq, seq[:, None] * seq[None, :]


def _err(got, ref):
    return oracle.relative_error(got.float().cpu(), ref)


@pytest.mark.parametrize("batch,m,n,k", [(1, 70, 33, 19), (3, 128, 130, 64)])
def test_f32_gemm_strided_with_epilogue(batch, m, n, k):
    g = torch.Generator().manual_seed(1)
    a = torch.randn(batch, k, m, generator=g)          # used transposed: a[b](i, k) = a[b, k, i]
    b = torch.randn(batch, n, k, generator=g)
    bias = torch.randn(n, generator=g)
    rs = torch.rand(batch, m, generator=g)
    mul = torch.randn(batch, m, n, generator=g)
    out = torch.empty(batch, m, n, device=DEV)
    fp32.gemm(a.to(DEV).transpose(1, 2), b.to(DEV), out, bias=bias.to(DEV), act=1,
              row_scale=rs.to(DEV), mul=mul.to(DEV))
    ref = torch.sigmoid(a.transpose(1, 2) @ b.transpose(1, 2) + bias) * rs[..., None] * mul
    assert _err(out, ref) < 1e-5


def test_f32_attention_edges():
    """Fully masked rows average every key; a NaN logit makes its row NaN; the
    bias is added before the mask, as the reference's torch path."""
    bsz, h, q, kk, d = 3, 2, 20, 37, 24
    g = torch.Generator().manual_seed(2)
    qt, kt, vt = (torch.randn(bsz, h, n, d, generator=g) for n in (q, kk, kk))
    bias = torch.randn(h, q, kk, generator=g)
    mask = (torch.rand(bsz, kk, generator=g) > 0.3).float()
    mask[1] = 0
    bias[1, 3, 5] = float("nan")
    out = torch.empty(bsz, h, q, d, device=DEV)
    fp32.attention(qt.to(DEV), kt.to(DEV), vt.to(DEV), out, bias=bias.to(DEV)[None],
                   mask=mask.to(DEV))
    ref = oracle.dot_product_attention(qt, kt, vt, mask=mask, bias=bias[None])
    got = out.cpu()
    assert torch.equal(torch.isnan(got), torch.isnan(ref))
    fin = ~torch.isnan(ref)
    assert oracle.relative_error(got[fin], ref[fin]) < 1e-5


@pytest.mark.parametrize("outgoing", [True, False])
def test_triangle_multiplication_fp32(outgoing):
    n = 72
    mod = TriangleMultiplication(128, _outgoing=outgoing).eval()
    init_params_(mod, seed=3, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(4)
    pair = torch.randn(n, n, 128, generator=g)
    _, pmask = _masks(n, 4)
    ref = oracle.triangle_multiplication(pair, pmask, _params(mod), outgoing)
    mod = mod.to(DEV)
    with torch.inference_mode():
        upd = mod(pair.to(DEV), pmask.to(DEV))
    assert upd.dtype == torch.float32
    assert _err(upd, ref) < TOL


@pytest.mark.parametrize("transpose", [False, True])
def test_grid_self_attention_fp32(transpose):
    n = 50
    mod = GridSelfAttention(128, 4, transpose=transpose).eval()
    init_params_(mod, seed=5, std=0.05, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(6)
    pair = torch.randn(n, n, 128, generator=g)
    _, pmask = _masks(n, 6)
    ref = oracle.grid_self_attention(pair, pmask, _params(mod), transpose, 4)
    mod = mod.to(DEV)
    with torch.inference_mode():
        upd = mod(pair.to(DEV), pmask.to(DEV))
    assert _err(upd, ref) < TOL


def test_transition_fp32():
    mod = Transition(128, 4).eval()
    init_params_(mod, seed=7, perturb_layer_norm=True)
    x = torch.randn(300, 128, generator=torch.Generator().manual_seed(8))
    ref = oracle.transition(x, _params(mod))
    with torch.inference_mode():
        upd = mod.to(DEV)(x.to(DEV))
    assert _err(upd, ref) < TOL


def test_conditioned_self_attention_and_transition_fp32():
    n, c = 64, 768
    att = SelfAttention(c, 384, 16, use_single_cond=True).eval()
    tr = DiffusionTransition(c, 384, 2, use_single_cond=True).eval()
    init_params_(att, seed=9, std=0.05, perturb_layer_norm=True)
    init_params_(tr, seed=10, std=0.05, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(n, c, generator=g)
    cond = torch.randn(n, 384, generator=g)
    logits = torch.randn(16, n, n, generator=g)
    seq, _ = _masks(n, 3)
    ref_a = oracle.self_attention(x, seq, logits, _params(att), cond, 16, True)
    ref_t = oracle.diffusion_transition(x, cond, _params(tr), True)
    with torch.inference_mode():
        upd_a = att.to(DEV)(x.to(DEV), seq.to(DEV), logits.to(DEV), cond.to(DEV))
        upd_t = tr.to(DEV)(x.to(DEV), cond.to(DEV))
    assert _err(upd_a, ref_a) < TOL
    assert _err(upd_t, ref_t) < TOL


def test_pairformer_block_fp32():
    n = 48
    block = PairformerBlock().eval()
    init_params_(block, seed=12, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(13)
    pair = torch.randn(n, n, 128, generator=g)
    single = torch.randn(n, 384, generator=g)
    seq, pmask = _masks(n, 5)
    ref_p, ref_s = oracle.pairformer_block(pair, pmask, single, seq, _params(block))
    block = block.to(DEV)
    p, s = pair.to(DEV), single.to(DEV)
    with torch.inference_mode():
        block(p, pmask.to(DEV), s, seq.to(DEV))
    assert _err(p - pair.to(DEV), ref_p - pair) < TOL
    assert _err(s - single.to(DEV), ref_s - single) < TOL


def test_diffusion_transformer_fp32():
    n, c = 40, 768
    mod = DiffusionTransformer(c_act=c, num_blocks=4, super_block_size=2).eval()
    init_params_(mod, seed=14, std=0.05, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(15)
    act = torch.randn(n, c, generator=g)
    cond = torch.randn(n, 384, generator=g)
    pair_cond = torch.randn(n, n, 128, generator=g)
    seq, _ = _masks(n, 2)
    ref = oracle.diffusion_transformer(act, seq, cond, pair_cond, _params(mod), num_blocks=4,
                                       super_block_size=2)
    a = act.to(DEV)
    with torch.inference_mode():
        mod.to(DEV)(a, seq.to(DEV), cond.to(DEV), pair_cond.to(DEV))
    assert _err(a - act.to(DEV), ref - act) < TOL


def test_small_triangle_directions_fp32():
    """The reference's own small-case check (3 tokens, c = 8, an identity mask;
    tests/test_cpu_runtime.py:104-115 of the reference): each direction equals
    the explicit per-channel contraction, in float32."""
    for outgoing in (False, True):
        mod = TriangleMultiplication(8, _outgoing=outgoing).eval()
        init_params_(mod, seed=21, std=0.3, perturb_layer_norm=True)
        g = torch.Generator().manual_seed(22)
        pair, mask = torch.randn(3, 3, 8, generator=g), torch.eye(3)
        p = {k: v.detach().float() for k, v in mod.state_dict().items()}
        with torch.no_grad():
            x = torch.nn.functional.layer_norm(pair, (8,), p["left_norm_input.weight"],
                                               p["left_norm_input.bias"])
            proj = (x @ p["projection.weight"].T) * mask[..., None] * torch.sigmoid(
                x @ p["gate.weight"].T)
            a, b = proj[..., 0::2], proj[..., 1::2]
            prod = torch.stack([a[..., c] @ b[..., c].T if outgoing else b[..., c].T @ a[..., c]
                                for c in range(8)], dim=-1)
            z = torch.nn.functional.layer_norm(prod, (8,), p["center_norm.weight"],
                                               p["center_norm.bias"])
            want = (z @ p["output_projection.weight"].T) * torch.sigmoid(
                x @ p["gating_linear.weight"].T)
        with torch.inference_mode():
            got = mod.to(DEV)(pair.to(DEV), mask.to(DEV))
        assert _err(got, want) < 1e-5


def test_small_pairformer_block_fp32():
    """3 tokens, c_pair = c_single = 8, two heads each (the reference's
    end-to-end smoke shape, tests/test_cpu_runtime.py:117-125), against the
    float32 oracle."""
    block = PairformerBlock(n_heads=2, c_pair=8, c_single=8, n_heads_pair=2).eval()
    init_params_(block, seed=23, std=0.3, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(24)
    pair, single = torch.randn(3, 3, 8, generator=g), torch.randn(3, 8, generator=g)
    ref_p, ref_s = oracle.pairformer_block(pair, torch.ones(3, 3), single, torch.ones(3),
                                           _params(block), n_heads=2, n_heads_pair=2)
    block = block.to(DEV)
    p, s = pair.to(DEV), single.to(DEV)
    with torch.inference_mode():
        block(p, torch.ones(3, 3, device=DEV), s, torch.ones(3, device=DEV))
    assert torch.isfinite(p).all() and torch.isfinite(s).all()
    assert _err(p - pair.to(DEV), ref_p - pair) < TOL
    assert _err(s - single.to(DEV), ref_s - single) < TOL


def test_f32_layer_norm_matches_torch():
    g = torch.Generator(device="cuda").manual_seed(25)
    for c in (8, 128, 384, 768):
        x = torch.randn(257, c, device=DEV, generator=g) * 3 + 1
        w = torch.randn(c, device=DEV, generator=g)
        b = torch.randn(c, device=DEV, generator=g)
        got = fp32.layer_norm(x, w, b, 1e-5)
        want = torch.nn.functional.layer_norm(x, (c,), w, b, 1e-5)
        assert oracle.relative_error(got.cpu(), want.cpu()) < 1e-5
