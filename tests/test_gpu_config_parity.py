"""Parity of the CUDA path with the CPU oracle at the BASELINE configurations.

C2: TriangleMultiplication outgoing and incoming, N in {256, 512, 768, 1024,
    1536}, bf16 activations, z ~ N(0, 1), weights ~ N(0, 0.02) (LayerNorm
    gamma = 1, beta = 0), the last ceil(0.05 N) rows and columns of the pair
    mask zero, seed 1.
C3: GridSelfAttention around the starting and the ending node, N in {512,
    1024, 2048}, 4 heads of 32, key mask with a padded tail of 64 tokens, seed 2.
C4: one Pairformer block at N = 1024 (c_pair 128, c_single 384), seed 3,
    checked operator by operator: each update of the pair is compared with the
    oracle applied to the same input, so an error cannot hide behind the
    residual stream.

The oracle evaluates sampled output rows (oracle.triangle_multiplication_rows,
oracle.grid_self_attention_rows; equal to the full restatement up to float32
summation order, see tests/test_oracle_golden.py), chosen to cover the first rows, the middle, the
last unmasked row, the first masked row and the last row.  Tolerance: max
|got - ref| / max |ref| <= 1e-2 over the sampled rows of the update, the bf16
bar of the north star.  Also here: the attention edge semantics of the
reference's native kernel (af3_kernels/src/csrc/dot_product_attention.cpp:
a NaN logit makes its query row NaN unless the key is masked, :72-88; an empty
key set returns zeros, :141-144).
"""

import math

import pytest
import torch

import oracle
from xfold_cpu_b200 import _capi, native

pytestmark = pytest.mark.gpu

TOL = 1e-2
DEV = "cuda"
C = 128


@pytest.fixture(autouse=True)
def _no_device_error():
    _capi.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert _capi.device_error(clear=True) == 0


def _sample_rows(n: int, tail: int) -> list[int]:
    rows = {0, 1, n // 3, n // 2 + 7, n - tail - 1, n - tail, n - 1}
    return sorted(r for r in rows if 0 <= r < n)


def _pair_mask(n: int, tail: int) -> torch.Tensor:
    m = torch.ones(n)
    m[n - tail:] = 0
    return m[:, None] * m[None, :]


def _rel_rows(got_rows: torch.Tensor, ref_rows: torch.Tensor) -> float:
    return oracle.relative_error(got_rows.float().cpu(), ref_rows)


# ----------------------------------------------------------------------------- C2

def _c2_params(g: torch.Generator) -> dict:
    w = lambda *s: torch.randn(*s, generator=g) * 0.02
    return {"left_norm_input.weight": torch.ones(C), "left_norm_input.bias": torch.zeros(C),
            "projection.weight": w(2 * C, C), "gate.weight": w(2 * C, C),
            "center_norm.weight": torch.ones(C), "center_norm.bias": torch.zeros(C),
            "output_projection.weight": w(C, C), "gating_linear.weight": w(C, C)}


@pytest.mark.parametrize("outgoing", [True, False], ids=["outgoing", "incoming"])
@pytest.mark.parametrize("n", [256, 512, 768, 1024, 1536])
def test_c2_triangle_multiplication(n, outgoing):
    g = torch.Generator().manual_seed(1)
    pair = torch.randn(n, n, C, generator=g).bfloat16()
    p = _c2_params(g)
    tail = math.ceil(0.05 * n)
    mask = _pair_mask(n, tail)
    rows = _sample_rows(n, tail)
    d = {k: v.to(DEV) for k, v in p.items()}
    got = native.triangle_multiplication(
        pair.to(DEV), mask.to(DEV), outgoing, d["left_norm_input.weight"],
        d["left_norm_input.bias"], d["projection.weight"], d["gate.weight"],
        d["center_norm.weight"], d["center_norm.bias"], d["output_projection.weight"],
        d["gating_linear.weight"], out_dtype=torch.float32)
    got_rows = got[rows].cpu()
    assert torch.isfinite(got).all()
    del got
    ref = oracle.triangle_multiplication_rows(pair.float(), mask, p, outgoing, rows)
    assert _rel_rows(got_rows, ref) < TOL


# ----------------------------------------------------------------------------- C3

def _c3_params(g: torch.Generator) -> dict:
    w = lambda *s: torch.randn(*s, generator=g) * 0.02
    return {"act_norm.weight": torch.ones(C), "act_norm.bias": torch.zeros(C),
            "pair_bias_projection.weight": w(4, C), "q_projection.weight": w(C, C),
            "k_projection.weight": w(C, C), "v_projection.weight": w(C, C),
            "gating_query.weight": w(C, C), "output_projection.weight": w(C, C)}


@pytest.mark.parametrize("transpose", [False, True], ids=["starting", "ending"])
@pytest.mark.parametrize("n", [512, 1024, 2048])
def test_c3_grid_self_attention(n, transpose):
    g = torch.Generator().manual_seed(2)
    pair = torch.randn(n, n, C, generator=g).bfloat16()
    p = _c3_params(g)
    mask = _pair_mask(n, 64)
    rows = _sample_rows(n, 64)
    d = {k: v.to(DEV) for k, v in p.items()}
    packed = native.pack_attention_weights(d["q_projection.weight"], d["k_projection.weight"],
                                           d["v_projection.weight"], d["gating_query.weight"])
    got = native.grid_self_attention(pair.to(DEV), mask.to(DEV), transpose, d["act_norm.weight"],
                                     d["act_norm.bias"], 1e-5, d["pair_bias_projection.weight"],
                                     packed, d["output_projection.weight"], 4,
                                     out_dtype=torch.float32)
    got_rows = (got[:, rows].permute(1, 0, 2) if transpose else got[rows]).cpu()
    assert torch.isfinite(got).all()
    del got
    ref = oracle.grid_self_attention_rows(pair.float(), mask, p, transpose, rows, 4)
    assert _rel_rows(got_rows, ref) < TOL


# ----------------------------------------------------------------------------- C4

def test_c4_pairformer_block_operator_by_operator():
    from xfold_cpu_b200.nn import PairformerBlock, init_params_

    n = 1024
    g = torch.Generator().manual_seed(3)
    pair_h = torch.randn(n, n, C, generator=g)
    single_h = torch.randn(n, 384, generator=g)
    seq = torch.ones(n)
    seq[n - 64:] = 0
    pair_mask_h = seq[:, None] * seq[None, :]
    blk = PairformerBlock(c_pair=C, c_single=384).eval()
    init_params_(blk, seed=3000)
    params = {k: v.detach().clone() for k, v in blk.state_dict().items()}
    blk = blk.to(DEV)
    rows = _sample_rows(n, 64)
    pair, pair_mask = pair_h.to(DEV), pair_mask_h.to(DEV)
    single, seq_mask = single_h.to(DEV), seq.to(DEV)
    errors = {}
    with torch.inference_mode():
        stages = [
            ("triangle_multiplication_outgoing", blk.triangle_multiplication_outgoing,
             lambda x: oracle.triangle_multiplication_rows(
                 x, pair_mask_h, params, True, rows, "triangle_multiplication_outgoing.")),
            ("triangle_multiplication_incoming", blk.triangle_multiplication_incoming,
             lambda x: oracle.triangle_multiplication_rows(
                 x, pair_mask_h, params, False, rows, "triangle_multiplication_incoming.")),
            ("pair_attention1", blk.pair_attention1,
             lambda x: oracle.grid_self_attention_rows(x, pair_mask_h, params, False, rows, 4,
                                                       "pair_attention1.")),
            ("pair_attention2", blk.pair_attention2,
             lambda x: oracle.grid_self_attention_rows(x, pair_mask_h, params, True, rows, 4,
                                                       "pair_attention2.")),
        ]
        for name, mod, ref_fn in stages:
            before = pair.clone()
            mod.accumulate_(pair, pair_mask)
            upd = pair - before
            got_rows = (upd[:, rows].permute(1, 0, 2) if name == "pair_attention2"
                        else upd[rows]).cpu()
            del upd
            errors[name] = _rel_rows(got_rows, ref_fn(before.cpu()))
            del before
        before = pair.clone()
        blk.pair_transition.accumulate_(pair)
        got_rows = (pair - before)[rows].cpu()
        errors["pair_transition"] = _rel_rows(
            got_rows, oracle.transition(before[rows].cpu(), params, "pair_transition."))
        del before
        # single track: logits from the updated pair, then attention and transition in full
        s0 = single.clone()
        norm = blk.single_pair_logits_norm
        logits = native.pair_logits(pair, norm.weight, norm.bias, norm.eps,
                                    blk.single_pair_logits_projection.weight.bfloat16())
        blk.single_attention_.accumulate_(single, seq_mask, logits)
        pair_cpu = pair.cpu()
        ref_logits = oracle.pair_logits(pair_cpu, params)
        errors["single_pair_logits"] = oracle.relative_error(logits.float().cpu(), ref_logits)
        ref_att = oracle.self_attention(s0.cpu(), seq, ref_logits, params, None, 16, False,
                                        "single_attention_.")
        errors["single_attention"] = oracle.relative_error((single - s0).cpu(), ref_att)
        s1 = single.clone()
        blk.single_transition.accumulate_(single)
        errors["single_transition"] = oracle.relative_error(
            (single - s1).cpu(), oracle.transition(s1.cpu(), params, "single_transition."))
    assert torch.isfinite(pair).all() and torch.isfinite(single).all()
    bad = {k: v for k, v in errors.items() if not v < TOL}
    assert not bad, f"update errors above {TOL}: {bad} (all: {errors})"


# ----------------------------------------------------------------------------- attention edges

@pytest.mark.parametrize("B", [2, 48])
def test_nan_and_infinite_bias_semantics(B):
    """The caller-facing attention keeps the reference's semantics for
    non-finite scores (dot_product_attention.cpp:72-88): a NaN score makes its
    query row NaN; a NaN at a masked key is replaced by -1e9 first and poisons
    nothing; a -inf bias gives its key probability 0 and leaves the row finite."""
    g = torch.Generator().manual_seed(9)
    H, n, d = 4, 128, 32
    q = torch.randn(B, H, n, d, generator=g) * 0.3
    k = torch.randn(B, H, n, d, generator=g) * 0.3
    v = torch.randn(B, H, n, d, generator=g)
    bias = torch.randn(1, H, n, n, generator=g).bfloat16()
    mask = torch.ones(B, n)
    mask[:, -8:] = 0
    q[0, 1, 5, 3] = float("nan")          # row (0, 1, 5): NaN logits everywhere
    k[1, 2, n - 3, 0] = float("nan")      # masked key: no effect
    bias[0, 3, 7, 11] = float("nan")      # row 7 of head 3, every batch row: NaN
    bias[0, 0, 9, 20] = float("-inf")     # key 20 of row 9, head 0: probability 0
    bias[0, 2, 4, n - 2] = float("nan")   # masked key: no effect
    out = native.dot_product_attention(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV),
                                       bias.to(DEV)).float().cpu()
    nan_rows = torch.isnan(out).any(dim=-1)
    expect = torch.zeros(B, H, n, dtype=torch.bool)
    expect[0, 1, 5] = True
    expect[:, 3, 7] = True
    assert torch.equal(nan_rows, expect)
    assert torch.isnan(out[0, 1, 5]).all() and torch.isnan(out[:, 3, 7]).all()
    ref = oracle.dot_product_attention(q, k, v, mask=mask, bias=bias.float())
    ok = ~expect
    assert torch.isfinite(ref[ok]).all()
    assert oracle.relative_error(out[ok], ref[ok]) < TOL


def test_triangle_attention_core_nan_row_and_masked_nan_key():
    """The three-slot triangle-attention kernel (48 or more rows sharing one
    bias): parity with the oracle, a NaN query poisons its own row and head
    only, a NaN key that is masked poisons nothing."""
    g = torch.Generator().manual_seed(10)
    rows, H, n = 50, 4, 192
    log2e = 1.4426950408889634
    q = torch.randn(rows, H, n, 32, generator=g) * 0.3
    k = torch.randn(rows, H, n, 32, generator=g) * 0.3
    v = torch.randn(rows, H, n, 32, generator=g)
    bias = torch.randn(H, n, n, generator=g)
    gate = torch.rand(rows, n, H * 32, generator=g)
    mask = torch.ones(rows, n)
    mask[:, -16:] = 0
    mask[7] = 0  # a fully masked row: uniform attention
    q[3, 1, 5, 0] = float("nan")
    k[4, 2, n - 1, 0] = float("nan")
    qs = (q * log2e / math.sqrt(32)).bfloat16()
    bs = (bias * log2e).bfloat16()
    out = native.grid_attention_core(qs.to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV),
                                     mask.to(DEV), bs.to(DEV), gate.bfloat16().to(DEV))
    out = out.float().cpu().reshape(rows, n, H, 32)
    nan_rows = torch.isnan(out).any(dim=-1)
    expect = torch.zeros(rows, n, H, dtype=torch.bool)
    expect[3, 5, 1] = True
    assert torch.equal(nan_rows, expect)
    qo = qs.float() / log2e * math.sqrt(32)  # the oracle scales q by d^-0.5 itself
    ref = oracle.dot_product_attention(qo, k.bfloat16().float(), v.bfloat16().float(), mask=mask,
                                       bias=(bs.float() / log2e)[None])
    ref = (ref.permute(0, 2, 1, 3) * gate.bfloat16().float().reshape(rows, n, H, 32))
    ok = ~expect
    assert oracle.relative_error(out[ok], ref[ok]) < TOL


def test_empty_key_set_returns_zeros():
    """No keys: the reference returns zeros (dot_product_attention.cpp:141-144)."""
    q = torch.randn(2, 3, 40, 32, device=DEV)
    k = torch.randn(2, 3, 0, 32, device=DEV)
    v = torch.randn(2, 3, 0, 32, device=DEV)
    out = native.dot_product_attention(q, k, v, torch.ones(2, 0, device=DEV))
    torch.cuda.synchronize()
    assert out.shape == (2, 3, 40, 32)
    assert torch.count_nonzero(out.float()) == 0


# ----------------------------------------------------------------------------- C5

def test_c5_diffusion_transformer_24_blocks():
    """C5's token transformer at full size: 24 blocks in 6 super-blocks, N = 768,
    c = 768, 16 heads of 48, single cond 384, pair cond [768, 768, 128], random
    init N(0, 0.02) with LayerNorm gamma 1 / beta 0, seed 4, 32 padded tokens;
    the update of one forward against the oracle of DiffusionTransformer.forward
    (xfold/nn/diffusion_transformer.py:250-272)."""
    from xfold_cpu_b200.nn import DiffusionTransformer, init_params_

    n, c = 768, 768
    mod = DiffusionTransformer(c_act=c).eval()
    init_params_(mod, seed=4)
    params = {k: v.detach().clone() for k, v in mod.state_dict().items()}
    g = torch.Generator().manual_seed(4)
    act = torch.randn(n, c, generator=g)
    cond = torch.randn(n, 384, generator=g)
    pair_cond = torch.randn(n, n, 128, generator=g)
    mask = torch.ones(n)
    mask[-32:] = 0
    mod = mod.to(DEV)
    got = act.to(DEV)
    with torch.inference_mode():
        mod(got, mask.to(DEV), cond.to(DEV), pair_cond.to(DEV))
    got = got.cpu()
    assert torch.isfinite(got).all()
    with torch.inference_mode():
        ref = oracle.diffusion_transformer(act, mask, cond, pair_cond, params)
    assert oracle.relative_error(got - act, ref - act) < TOL
