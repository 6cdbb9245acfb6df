"""Generates the golden fixtures of tests/golden/*.npz by running the
reference implementation itself (xfold, torch backend, CPU).

Usage (from the repository root, with the reference checkout available):
    PYTHONPATH=<xfold checkout> python tests/golden/make_golden.py [fixture ...]

With fixture names, only those files are written (the random stream is the
same, so every fixture is reproducible on its own).

Each fixture holds the inputs, the module's state_dict (parameter names of
the reference modules) and the reference outputs, in float32; `bf16:` entries
are the same forward under torch.amp.autocast('cpu', bfloat16), the precision
mode of the reference's GPU route.  Sizes are small so the files stay small;
the oracle tests replay them through oracle/hotpath.py.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _init(module: torch.nn.Module, seed: int, std: float = 0.2) -> None:
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            owner = module.get_submodule(name.rsplit(".", 1)[0]) if "." in name else module
            if isinstance(owner, torch.nn.Linear):
                p.copy_(torch.randn(p.shape, generator=g) * std)
            elif name.endswith("weight"):
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(0.1 * torch.randn(p.shape, generator=g))


ONLY: set[str] = set()  # fixture names given on the command line; empty = all


def _save(name: str, module, inputs: dict, outputs: dict) -> None:
    if ONLY and name not in ONLY:
        return
    arrays = {}
    if module is not None:
        for k, v in module.state_dict().items():
            arrays[f"param:{k}"] = v.detach().float().numpy()
    for k, v in inputs.items():
        arrays[f"in:{k}"] = v.detach().float().numpy()
    for k, v in outputs.items():
        arrays[f"out:{k}"] = v.detach().float().numpy()
    np.savez_compressed(OUT / f"{name}.npz", **arrays)
    print(f"wrote {name}.npz ({sum(a.size for a in arrays.values())} values)")


def _both(fn):
    """Runs fn() in float32 and under CPU bf16 autocast (inference mode)."""
    with torch.inference_mode():
        fp32 = fn()
        with torch.amp.autocast("cpu", dtype=torch.bfloat16):
            bf16 = fn()
    return fp32, bf16


def main() -> None:
    from xfold.fastnn import config
    from xfold import fastnn
    from xfold.nn.attention import GridSelfAttention
    from xfold.nn.diffusion_transformer import DiffusionTransition, SelfAttention
    from xfold.nn.pairformer import PairformerBlock
    from xfold.nn.primitives import Transition
    from xfold.nn.triangle_multiplication import TriangleMultiplication

    for opt in ("layer_norm_implementation", "dot_product_attention_implementation",
                "gated_linear_unit_implementation", "triangle_multiplication_implementation"):
        setattr(config, opt, "torch")
    g = torch.Generator().manual_seed(1234)

    def masks(n, tail):
        seq = torch.ones(n)
        seq[-tail:] = 0
        return seq, seq[:, None] * seq[None, :]

    # --- TriangleMultiplication, both directions, ragged mask (reference test :104-115 pattern)
    for outgoing in (True, False):
        n, c = 9, 16
        mod = TriangleMultiplication(c, _outgoing=outgoing).eval()
        _init(mod, 10 + outgoing)
        pair = torch.randn(n, n, c, generator=g)
        mask = (torch.rand(n, n, generator=g) > 0.2).float()
        fp32, bf16 = _both(lambda: mod(pair, mask))
        _save(f"triangle_{'outgoing' if outgoing else 'incoming'}", mod,
              {"pair": pair, "mask": mask}, {"update": fp32, "bf16:update": bf16})

    # --- GridSelfAttention, starting and ending node
    for transpose in (False, True):
        n, c = 7, 16
        mod = GridSelfAttention(c, num_head=4, transpose=transpose).eval()
        _init(mod, 20 + transpose)
        pair = torch.randn(n, n, c, generator=g)
        _, mask = masks(n, 2)
        fp32, bf16 = _both(lambda: mod(pair, mask))
        _save(f"grid_attention_{'ending' if transpose else 'starting'}", mod,
              {"pair": pair, "mask": mask}, {"update": fp32, "bf16:update": bf16})

    # --- Transition (GLU)
    mod = Transition(16, num_intermediate_factor=4).eval()
    _init(mod, 30)
    x = torch.randn(5, 6, 16, generator=g)
    fp32, bf16 = _both(lambda: mod(x))
    _save("transition", mod, {"x": x}, {"update": fp32, "bf16:update": bf16})

    # --- dot_product_attention with mask ranks 1/2/4 and bias (reference test :70-89 pattern)
    q = torch.randn(2, 3, 5, 8, generator=g)
    k = torch.randn(2, 3, 6, 8, generator=g)
    v = torch.randn(2, 3, 6, 8, generator=g)
    bias = torch.randn(2, 3, 5, 6, generator=g)
    m1 = torch.tensor([1, 1, 0, 1, 0, 1], dtype=torch.bool)
    m2 = torch.tensor([[1, 0, 1, 1, 1, 0], [0, 0, 0, 0, 0, 0]], dtype=torch.bool)
    m4 = m1[None, None, None, :].expand(2, 1, 1, 6)
    outs = {}
    with torch.inference_mode():
        for tag, mask in (("rank1", m1), ("rank2", m2), ("rank4", m4), ("none", None)):
            outs[tag] = fastnn.dot_product_attention(q, k, v, mask=mask, bias=bias)
    _save("dot_product_attention", None,
          {"q": q, "k": k, "v": v, "bias": bias, "mask_rank1": m1.float(), "mask_rank2": m2.float(),
           "mask_rank4": m4.float()}, outs)

    # --- SelfAttention, plain (single track) and conditioned (diffusion)
    for cond in (False, True):
        n, c, cs = 10, 32, 8
        mod = SelfAttention(c, cs, num_head=4, use_single_cond=cond).eval()
        _init(mod, 40 + cond)
        x = torch.randn(n, c, generator=g)
        seq, _ = masks(n, 3)
        logits = torch.randn(4, n, n, generator=g)
        sc = torch.randn(n, cs, generator=g) if cond else None
        fp32, bf16 = _both(lambda: mod(x, seq, logits, sc))
        inputs = {"x": x, "mask": seq, "pair_logits": logits}
        if cond:
            inputs["single_cond"] = sc
        _save(f"self_attention_{'conditioned' if cond else 'plain'}", mod, inputs,
              {"update": fp32, "bf16:update": bf16})

    # --- DiffusionTransition (conditioned)
    mod = DiffusionTransition(16, 8, use_single_cond=True).eval()
    _init(mod, 50)
    x = torch.randn(6, 16, generator=g)
    sc = torch.randn(6, 8, generator=g)
    fp32, bf16 = _both(lambda: mod(x, sc))
    _save("diffusion_transition", mod, {"x": x, "single_cond": sc},
          {"update": fp32, "bf16:update": bf16})

    # --- PairformerBlock end to end (reference test :117-125 pattern)
    n = 8
    mod = PairformerBlock(n_heads=4, c_pair=16, c_single=32, n_heads_pair=4).eval()
    _init(mod, 60, std=0.1)
    pair = torch.randn(n, n, 16, generator=g)
    single = torch.randn(n, 32, generator=g)
    seq, pmask = masks(n, 2)

    def block():
        p, s = pair.clone(), single.clone()
        return mod(p, pmask, s, seq)

    (p32, s32), (p16, s16) = _both(block)
    _save("pairformer_block", mod, {"pair": pair, "single": single, "pair_mask": pmask, "seq_mask": seq},
          {"pair": p32, "single": s32, "bf16:pair": p16, "bf16:single": s16})

    # --- CrossAttention of the atom transformer (small widths), masked queries
    # and keys so that the 1e9 * !mask_q * !mask_k term of the reference is hit
    from xfold.nn.atom_layout import GatherInfo
    from xfold.nn.diffusion_transformer import CrossAttention, DiffusionCrossAttTransformer

    s_, nq, nk, c, cs = 3, 4, 6, 16, 16  # the reference ties AdaLNZero's width to key_dim
    mod = CrossAttention(key_dim=c, value_dim=c, c_single_cond=cs, num_head=4).eval()
    _init(mod, 70)
    x_q = torch.randn(s_, nq, c, generator=g)
    x_k = torch.randn(s_, nk, c, generator=g)
    mask_q = torch.rand(s_, nq, generator=g) > 0.3
    mask_k = torch.rand(s_, nk, generator=g) > 0.3
    mask_q[0, -1] = False
    mask_k[0, -2:] = False
    logits = torch.randn(s_, 4, nq, nk, generator=g)
    scq = torch.randn(s_, nq, cs, generator=g)
    sck = torch.randn(s_, nk, cs, generator=g)
    fp32, bf16 = _both(lambda: mod(x_q, x_k, mask_q, mask_k, logits, scq, sck))
    _save("cross_attention", mod,
          {"x_q": x_q, "x_k": x_k, "mask_q": mask_q.float(), "mask_k": mask_k.float(),
           "pair_logits": logits, "single_cond_q": scq, "single_cond_k": sck},
          {"update": fp32, "bf16:update": bf16})

    # --- DiffusionCrossAttTransformer: the reference's own forward (pair logits
    # with two blocks, per-block key gather, residual updates) with its
    # cross-attention modules swapped for small-width ones
    nb = 2
    mod = DiffusionCrossAttTransformer(c_query=c, c_single_cond=cs, c_pair_cond=16,
                                       num_blocks=nb, num_head=4).eval()
    mod.cross_attention = torch.nn.ModuleList(
        [CrossAttention(key_dim=c, value_dim=c, c_single_cond=cs, num_head=4) for _ in range(nb)])
    _init(mod, 80)
    act = torch.randn(s_, nq, c, generator=g)
    q_mask = torch.rand(s_, nq, generator=g) > 0.2
    q_mask[-1, -1] = False
    idx = torch.randint(0, s_ * nq, (s_, nk), generator=g)
    gmask = torch.rand(s_, nk, generator=g) > 0.2
    k_mask = q_mask.reshape(-1)[idx] & gmask
    qsc = torch.randn(s_, nq, cs, generator=g)
    ksc = torch.randn(s_, nk, cs, generator=g)
    pair_cond = torch.randn(s_, nq, nk, 16, generator=g)
    info = GatherInfo(gather_idxs=idx, gather_mask=gmask,
                      input_shape=torch.tensor((s_, nq)))

    def transformer():
        mod._input_cache = type(mod._input_cache)()
        return mod(act.clone(), q_mask, info, k_mask, qsc, ksc, pair_cond)

    fp32, bf16 = _both(transformer)
    _save("diffusion_cross_att_transformer", mod,
          {"queries_act": act, "queries_mask": q_mask.float(), "gather_idxs": idx.float(),
           "gather_mask": gmask.float(), "keys_mask": k_mask.float(),
           "queries_single_cond": qsc, "keys_single_cond": ksc, "pair_cond": pair_cond},
          {"queries_act": fp32, "bf16:queries_act": bf16})

    # --- MSA stack (Evoformer): MSAAttention at its own widths, a token masked in
    # every sequence (the key mask), OuterProductMean, and a whole EvoformerBlock
    # with c_pair = 16
    from xfold.nn.attention import MSAAttention
    from xfold.nn.pairformer import EvoformerBlock
    from xfold.nn.primitives import OuterProductMean

    s_, n_ = 5, 6
    mod = MSAAttention(c_msa=64, c_pair=128, num_head=8).eval()
    _init(mod, 90)
    msa = torch.randn(s_, n_, 64, generator=g)
    msa_mask = (torch.rand(s_, n_, generator=g) > 0.25).float()
    msa_mask[:, 2] = 0.0
    pair = torch.randn(n_, n_, 128, generator=g)
    fp32, bf16 = _both(lambda: mod(msa, msa_mask, pair))
    _save("msa_attention", mod, {"msa": msa, "msa_mask": msa_mask, "pair": pair},
          {"update": fp32, "bf16:update": bf16})

    mod = OuterProductMean(c_msa=64, num_output_channel=16).eval()
    _init(mod, 91)
    with torch.no_grad():  # output_w / output_b are plain Parameters: small values
        mod.output_w.mul_(0.1)
        mod.output_b.mul_(0.1)
    msa = torch.randn(s_, n_, 64, generator=g)
    fp32, bf16 = _both(lambda: mod(msa, msa_mask))
    _save("outer_product_mean", mod, {"msa": msa, "mask": msa_mask},
          {"update": fp32, "bf16:update": bf16})

    mod = EvoformerBlock(c_msa=64, c_pair=16, n_heads_pair=4).eval()
    _init(mod, 92, std=0.1)
    with torch.no_grad():
        mod.outer_product_mean.output_w.mul_(0.1)
    msa = torch.randn(s_, n_, 64, generator=g)
    pair = torch.randn(n_, n_, 16, generator=g)
    _, pmask = masks(n_, 1)

    def evo():
        m, p = msa.clone(), pair.clone()
        return mod(m, p, msa_mask, pmask)

    (m32, p32), (m16, p16) = _both(evo)
    _save("evoformer_block", mod, {"msa": msa, "pair": pair, "msa_mask": msa_mask, "pair_mask": pmask},
          {"msa": m32, "pair": p32, "bf16:msa": m16, "bf16:pair": p16})


def diffusion_transformer_fixture() -> None:
    """DiffusionTransformer.forward (diffusion_transformer.py:250-272): 4 blocks in
    2 super-blocks, c_act 64, single cond 32, pair cond 8, masked tail; 16
    heads (of 4), since the reference builds its SelfAttention with the default
    head count (:243-244); its own random stream so the other fixtures are
    unchanged."""
    from xfold.nn.diffusion_transformer import DiffusionTransformer

    g = torch.Generator().manual_seed(4321)
    n = 16
    mod = DiffusionTransformer(c_act=64, c_single_cond=32, c_pair_cond=8, num_head=16,
                               num_blocks=4, super_block_size=2).eval()
    _init(mod, 95, std=0.1)
    act = torch.randn(n, 64, generator=g)
    sc = torch.randn(n, 32, generator=g)
    pc = torch.randn(n, n, 8, generator=g)
    mask = torch.ones(n)
    mask[-3:] = 0
    fp32, bf16 = _both(lambda: mod(act.clone(), mask, sc, pc))
    _save("diffusion_transformer", mod,
          {"act": act, "mask": mask, "single_cond": sc, "pair_cond": pc},
          {"act": fp32, "bf16:act": bf16})


if __name__ == "__main__":
    ONLY.update(sys.argv[1:])
    main()
    diffusion_transformer_fixture()
