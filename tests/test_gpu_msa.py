"""Evoformer MSA-stack parity on the GPU: MSAAttention, OuterProductMean and a
whole EvoformerBlock of the `cuda` backend against the CPU oracle (bf16 path
vs float32 oracle, tolerance 1e-2 on the update, max|delta| / max|ref|)."""

import pytest
import torch

import oracle
from xfold_cpu_b200 import _capi
from xfold_cpu_b200.nn import EvoformerBlock, MSAAttention, OuterProductMean, init_params_

pytestmark = pytest.mark.gpu

TOL = 1e-2
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _no_device_error():
    _capi.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert _capi.device_error(clear=True) == 0


def _params(module):
    return {k: v.detach().cpu().clone() for k, v in module.state_dict().items()}


def _msa_mask(s, n, seed, dead_token=None):
    g = torch.Generator().manual_seed(seed)
    mask = (torch.rand(s, n, generator=g) > 0.15).float()
    mask[0] = 1.0  # the query row of an MSA
    if dead_token is not None:
        mask[:, dead_token] = 0.0
    return mask


@pytest.mark.parametrize("s,n", [(16, 40), (5, 128)])
def test_msa_attention_module(s, n):
    mod = MSAAttention().eval()
    init_params_(mod, seed=60, std=0.1, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(61)
    msa = torch.randn(s, n, 64, generator=g)
    pair = torch.randn(n, n, 128, generator=g)
    mask = _msa_mask(s, n, 62, dead_token=n - 3)
    ref = oracle.msa_attention(msa, mask, pair, _params(mod))
    mod = mod.to(DEV)
    with torch.inference_mode():
        upd = mod(msa.to(DEV), mask.to(DEV), pair.to(DEV))
        assert upd.shape == msa.shape and upd.dtype == torch.bfloat16
        assert oracle.relative_error(upd.float().cpu(), ref) < TOL
        m = msa.to(DEV)
        mod.accumulate_(m, mask.to(DEV), pair.to(DEV))
    assert oracle.relative_error(m.cpu() - msa, ref) < TOL


@pytest.mark.parametrize("s,n", [(24, 48), (8, 200), (16, 256)])
def test_outer_product_mean_module(s, n):
    """n = 200 and 256 take two chunks of rows (a ragged and an even split)."""
    mod = OuterProductMean().eval()
    init_params_(mod, seed=63, std=0.1, perturb_layer_norm=True)
    with torch.no_grad():
        mod.output_w.copy_(torch.randn(mod.output_w.shape, generator=torch.Generator().manual_seed(1)) * 0.05)
        mod.output_b.copy_(torch.randn(128, generator=torch.Generator().manual_seed(2)) * 0.1)
    g = torch.Generator().manual_seed(64)
    msa = torch.randn(s, n, 64, generator=g)
    mask = _msa_mask(s, n, 65, dead_token=1)
    ref = oracle.outer_product_mean(msa, mask, _params(mod))
    mod = mod.to(DEV)
    with torch.inference_mode():
        upd = mod(msa.to(DEV), mask.to(DEV))
        assert upd.shape == (n, n, 128) and upd.dtype == torch.float32
        assert oracle.relative_error(upd.cpu(), ref) < TOL
        base = torch.randn(n, n, 128, generator=g)
        p = base.to(DEV)
        mod.accumulate_(p, msa.to(DEV), mask.to(DEV))
    assert oracle.relative_error(p.cpu() - base, ref) < TOL


def test_evoformer_block():
    s, n = 16, 48
    blk = EvoformerBlock().eval()
    init_params_(blk, seed=66, std=0.05, perturb_layer_norm=True)
    with torch.no_grad():
        blk.outer_product_mean.output_w.mul_(0.05)
        blk.outer_product_mean.output_b.mul_(0.05)
    g = torch.Generator().manual_seed(67)
    msa = torch.randn(s, n, 64, generator=g)
    pair = torch.randn(n, n, 128, generator=g)
    mask = _msa_mask(s, n, 68)
    seq = torch.ones(n)
    seq[-3:] = 0
    pmask = seq[:, None] * seq[None, :]
    ref_m, ref_p = oracle.evoformer_block(msa, pair, mask, pmask, _params(blk))
    blk = blk.to(DEV)
    m, p = msa.to(DEV), pair.to(DEV)
    with torch.inference_mode():
        out_m, out_p = blk(m, p, mask.to(DEV), pmask.to(DEV))
    assert out_m is m and out_p is p
    assert oracle.relative_error(m.cpu() - msa, ref_m - msa) < TOL
    assert oracle.relative_error(p.cpu() - pair, ref_p - pair) < TOL
