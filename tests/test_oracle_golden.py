"""Pins the CPU oracle to the reference: every golden fixture (made by running
the reference modules, tests/golden/make_golden.py) is replayed through
oracle/hotpath.py.  float32 outputs must agree to 1e-5 (relative to the
output's max magnitude); the reference's own bf16-autocast outputs are checked
to sit within the 1e-2 parity tolerance of the float32 oracle."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
FP32_TOL = 1e-5
BF16_TOL = 2e-2


def load(name):
    data = np.load(GOLDEN / f"{name}.npz")
    params = {k[6:]: torch.from_numpy(data[k]) for k in data.files if k.startswith("param:")}
    inputs = {k[3:]: torch.from_numpy(data[k]) for k in data.files if k.startswith("in:")}
    outputs = {k[4:]: torch.from_numpy(data[k]) for k in data.files if k.startswith("out:")}
    return params, inputs, outputs


def check(got, ref, tol):
    err = oracle.relative_error(got, ref)
    assert err <= tol, f"relative error {err:.3e} > {tol}"


@pytest.mark.parametrize("direction", ["outgoing", "incoming"])
def test_triangle_multiplication(direction):
    p, i, o = load(f"triangle_{direction}")
    got = oracle.triangle_multiplication(i["pair"], i["mask"], p, direction == "outgoing")
    check(got, o["update"], FP32_TOL)
    check(o["bf16:update"], got, BF16_TOL)


def test_triangle_direction_is_not_symmetric():
    """Planted mistake: swapping the contraction direction must be caught."""
    p, i, o = load("triangle_outgoing")
    wrong = oracle.triangle_multiplication(i["pair"], i["mask"], p, False)
    assert oracle.relative_error(wrong, o["update"]) > 1e-2


@pytest.mark.parametrize("node", ["starting", "ending"])
def test_grid_self_attention(node):
    p, i, o = load(f"grid_attention_{node}")
    got = oracle.grid_self_attention(i["pair"], i["mask"], p, node == "ending", 4)
    check(got, o["update"], FP32_TOL)
    check(o["bf16:update"], got, BF16_TOL)


def test_grid_attention_chunking_is_exact():
    p, i, o = load("grid_attention_ending")
    got = oracle.grid_self_attention(i["pair"], i["mask"], p, True, 4, batch_chunk=2)
    check(got, o["update"], FP32_TOL)


def test_transition():
    p, i, o = load("transition")
    got = oracle.transition(i["x"], p)
    check(got, o["update"], FP32_TOL)
    check(o["bf16:update"], got, BF16_TOL)


@pytest.mark.parametrize("rank", ["rank1", "rank2", "rank4", "none"])
def test_dot_product_attention(rank):
    _, i, o = load("dot_product_attention")
    mask = None
    if rank != "none":
        mask = i[f"mask_{rank}"].bool()
        if rank == "rank1" or rank == "rank2":
            mask = mask.float()
    got = oracle.dot_product_attention(i["q"], i["k"], i["v"], mask=mask, bias=i["bias"])
    check(got, o[rank], FP32_TOL)


def test_fully_masked_row_is_uniform():
    """rank2 fixture row 1 masks every key: the reference gives the plain mean of v."""
    _, i, o = load("dot_product_attention")
    mean_v = i["v"][1].mean(dim=1, keepdim=True).expand(-1, 5, -1)
    check(o["rank2"][1], mean_v, 1e-5)


@pytest.mark.parametrize("variant", ["plain", "conditioned"])
def test_self_attention(variant):
    p, i, o = load(f"self_attention_{variant}")
    cond = variant == "conditioned"
    got = oracle.self_attention(i["x"], i["mask"], i["pair_logits"], p, i.get("single_cond"), 4, cond)
    check(got, o["update"], FP32_TOL)
    check(o["bf16:update"], got, BF16_TOL)


def test_diffusion_transition():
    p, i, o = load("diffusion_transition")
    got = oracle.diffusion_transition(i["x"], i["single_cond"], p, True)
    check(got, o["update"], FP32_TOL)
    check(o["bf16:update"], got, BF16_TOL)


def test_pairformer_block():
    p, i, o = load("pairformer_block")
    pair, single = oracle.pairformer_block(i["pair"], i["pair_mask"], i["single"], i["seq_mask"], p,
                                           n_heads=4, n_heads_pair=4)
    check(pair, o["pair"], 1e-5)
    check(single, o["single"], 1e-5)
    check(o["bf16:pair"] - i["pair"], pair - i["pair"], BF16_TOL)
    check(o["bf16:single"] - i["single"], single - i["single"], BF16_TOL)


def _cross(p, i, mask_q=None, mask_k=None):
    return oracle.cross_attention(i["x_q"], i["x_k"],
                                  i["mask_q"].bool() if mask_q is None else mask_q,
                                  i["mask_k"].bool() if mask_k is None else mask_k,
                                  i["pair_logits"], p, i["single_cond_q"], i["single_cond_k"], 4)


def test_cross_attention():
    p, i, o = load("cross_attention")
    got = _cross(p, i)
    check(got, o["update"], FP32_TOL)
    check(o["bf16:update"], got, BF16_TOL)


def test_cross_attention_mask_term_is_pinned():
    """Planted mistake: without the reference's 1e9 * !mask_q * !mask_k term
    (all keys visible to every query, as the term leaves valid queries) the
    masked query rows change and the fixture catches it."""
    p, i, o = load("cross_attention")
    ones_q = torch.ones_like(i["mask_q"], dtype=torch.bool)
    wrong = _cross(p, i, mask_q=ones_q)
    assert oracle.relative_error(wrong, o["update"]) > 1e-2


def _cross_transformer(p, i, gather_idxs):
    return oracle.diffusion_cross_att_transformer(
        i["queries_act"], i["queries_mask"].bool(), gather_idxs, i["gather_mask"].bool(),
        i["keys_mask"].bool(), i["queries_single_cond"], i["keys_single_cond"], i["pair_cond"], p,
        num_blocks=2, num_head=4)


def test_diffusion_cross_att_transformer():
    p, i, o = load("diffusion_cross_att_transformer")
    got = _cross_transformer(p, i, i["gather_idxs"].long())
    check(got, o["queries_act"], FP32_TOL)
    check(o["bf16:queries_act"] - i["queries_act"], got - i["queries_act"], BF16_TOL)


def test_cross_att_transformer_gather_is_pinned():
    """Planted mistake: a shifted queries -> keys gather must be caught."""
    p, i, o = load("diffusion_cross_att_transformer")
    rows = i["queries_act"].shape[0] * i["queries_act"].shape[1]
    wrong = _cross_transformer(p, i, (i["gather_idxs"].long() + 1) % rows)
    assert oracle.relative_error(wrong, o["queries_act"]) > 1e-3


def test_msa_attention():
    p, i, o = load("msa_attention")
    got = oracle.msa_attention(i["msa"], i["msa_mask"], i["pair"], p, 8)
    check(got, o["update"], FP32_TOL)
    check(o["bf16:update"], got, BF16_TOL)


def test_msa_attention_key_mask_is_pinned():
    """Planted mistake: without the key mask (token 2 is masked in every
    sequence) the fixture catches the difference."""
    p, i, o = load("msa_attention")
    wrong = oracle.msa_attention(i["msa"], torch.ones_like(i["msa_mask"]), i["pair"], p, 8)
    assert oracle.relative_error(wrong, o["update"]) > 1e-2


def test_outer_product_mean():
    p, i, o = load("outer_product_mean")
    got = oracle.outer_product_mean(i["msa"], i["mask"], p)
    check(got, o["update"], FP32_TOL)
    check(o["bf16:update"], got, BF16_TOL)


def test_outer_product_mean_orientation_is_pinned():
    """Planted mistake: swapping the left and right projections transposes the
    outer product (i <-> j) and must be caught."""
    p, i, o = load("outer_product_mean")
    q = dict(p)
    q["left_projection.weight"], q["right_projection.weight"] = (p["right_projection.weight"],
                                                                 p["left_projection.weight"])
    wrong = oracle.outer_product_mean(i["msa"], i["mask"], q)
    assert oracle.relative_error(wrong, o["update"]) > 1e-2


def test_evoformer_block():
    p, i, o = load("evoformer_block")
    msa, pair = oracle.evoformer_block(i["msa"], i["pair"], i["msa_mask"], i["pair_mask"], p)
    check(msa, o["msa"], 1e-5)
    check(pair, o["pair"], 1e-5)
    check(o["bf16:msa"] - i["msa"], msa - i["msa"], BF16_TOL)
    check(o["bf16:pair"] - i["pair"], pair - i["pair"], BF16_TOL)


@pytest.mark.parametrize("outgoing", [True, False])
def test_sampled_row_triangle_multiplication_equals_the_full_restatement(outgoing):
    """oracle.triangle_multiplication_rows (used by the large-N GPU parity
    tests) gives the rows of oracle.triangle_multiplication, which the golden
    fixtures pin, up to float32 summation order (matrix products of other
    shapes); checked on the fixture's inputs."""
    name = "triangle_outgoing" if outgoing else "triangle_incoming"
    p, i, o = load(name)
    n = i["pair"].shape[0]
    rows = sorted({0, n // 2, n - 1})
    got = oracle.triangle_multiplication_rows(i["pair"], i["mask"], p, outgoing, rows, chunk=5)
    full = oracle.triangle_multiplication(i["pair"], i["mask"], p, outgoing)
    assert oracle.relative_error(got, full[rows]) < 1e-6
    check(got, o["update"][rows], FP32_TOL)


@pytest.mark.parametrize("transpose", [False, True])
def test_sampled_row_grid_attention_equals_the_full_restatement(transpose):
    name = "grid_attention_ending" if transpose else "grid_attention_starting"
    p, i, o = load(name)
    n = i["pair"].shape[0]
    rows = sorted({0, n // 2, n - 1})
    got = oracle.grid_self_attention_rows(i["pair"], i["mask"], p, transpose, rows, 4, chunk=7)
    full = oracle.grid_self_attention(i["pair"], i["mask"], p, transpose, 4)
    want = full[:, rows].permute(1, 0, 2) if transpose else full[rows]
    assert oracle.relative_error(got, want) < 1e-6
    ref = o["update"][:, rows].permute(1, 0, 2) if transpose else o["update"][rows]
    check(got, ref, FP32_TOL)


def test_diffusion_transformer():
    """The 24-block composition of DiffusionTransformer.forward (:250-272): the
    super-block pair-logit rearrangement and the residual order, on the
    reference's own output (4 blocks, 2 super-blocks)."""
    p, i, o = load("diffusion_transformer")
    got = oracle.diffusion_transformer(i["act"], i["mask"], i["single_cond"], i["pair_cond"], p,
                                       num_blocks=4, super_block_size=2, num_head=16)
    check(got, o["act"], 1e-5)
    check(o["bf16:act"] - i["act"], got - i["act"], BF16_TOL)


def test_diffusion_transformer_logit_layout_is_pinned():
    """Planted mistake: the super-block logits split as '(h b)' instead of
    '(b h)' must be caught."""
    p, i, o = load("diffusion_transformer")
    q = dict(p)
    for sb in range(2):
        w = p[f"pair_logits_projection.{sb}.weight"]  # rows (b h)
        q[f"pair_logits_projection.{sb}.weight"] = w.reshape(2, 16, -1).transpose(0, 1).reshape(w.shape)
    wrong = oracle.diffusion_transformer(i["act"], i["mask"], i["single_cond"], i["pair_cond"], q,
                                         num_blocks=4, super_block_size=2, num_head=16)
    assert oracle.relative_error(wrong - i["act"], o["act"] - i["act"]) > 1e-2
