"""Atom transformer parity on the GPU: the windowed cross-attention and
DiffusionCrossAttTransformer of the `cuda` backend against the CPU oracle
(bf16 path vs float32 oracle, tolerance 1e-2 on the update, max|delta| /
max|ref|), plus the fused key gather against explicitly gathered keys."""

import pytest
import torch

import oracle
from xfold_cpu_b200 import _capi
from xfold_cpu_b200.nn import CrossAttention, DiffusionCrossAttTransformer, GatherInfo, init_params_
from xfold_cpu_b200.nn import atom_layout

pytestmark = pytest.mark.gpu

TOL = 1e-2
DEV = torch.device("cuda")
NQ, NK, C = 32, 128, 128


@pytest.fixture(autouse=True)
def _no_device_error():
    _capi.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert _capi.device_error(clear=True) == 0


def _params(module):
    return {k: v.detach().cpu().clone() for k, v in module.state_dict().items()}


def windows(subsets: int, masked_tail: int):
    """Keys of subset s: the 128 query rows centred on its 32 queries (rows
    outside the atoms invalid), and the masks the encoder derives: the last
    `masked_tail` atoms masked, keys_mask = queries_mask gathered."""
    rows = subsets * NQ
    start = torch.arange(subsets)[:, None] * NQ + NQ // 2 - NK // 2
    idx = start + torch.arange(NK)[None, :]
    valid = (idx >= 0) & (idx < rows)
    idx = torch.where(valid, idx, torch.zeros_like(idx))
    qmask = torch.ones(rows, dtype=torch.bool)
    if masked_tail:
        qmask[-masked_tail:] = False
    kmask = qmask[idx] & valid
    info = GatherInfo(gather_idxs=idx, gather_mask=valid, input_shape=torch.tensor((subsets, NQ)))
    return info, qmask.reshape(subsets, NQ), kmask


def test_cross_pair_logits():
    s = 5
    mod = DiffusionCrossAttTransformer().eval()
    init_params_(mod, seed=31, std=0.3, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(32)
    pair_cond = torch.randn(s, NQ, NK, 16, generator=g)
    ref = oracle.cross_pair_logits(pair_cond, _params(mod), 3, 4)
    mod = mod.to(DEV)
    with torch.inference_mode():
        got = mod.pair_logits(pair_cond.to(DEV))
    assert got.shape == (3, s, 4, NQ, NK) and got.dtype == torch.bfloat16
    assert oracle.relative_error(got.float().cpu(), ref) < TOL


def _cross_inputs(s, seed):
    g = torch.Generator().manual_seed(seed)
    x_q = torch.randn(s, NQ, C, generator=g)
    x_k = torch.randn(s, NK, C, generator=g)
    mask_q = torch.rand(s, NQ, generator=g) > 0.2
    mask_k = torch.rand(s, NK, generator=g) > 0.2
    mask_q[0] = True  # a window with every query valid
    mask_k[1, :40] = False  # masked queries of window 1 see 40+ masked keys
    logits = torch.randn(s, 4, NQ, NK, generator=g).bfloat16().float()
    scq = torch.randn(s, NQ, C, generator=g)
    sck = torch.randn(s, NK, C, generator=g)
    return x_q, x_k, mask_q, mask_k, logits, scq, sck


def test_cross_attention_module():
    s = 6
    mod = CrossAttention().eval()
    init_params_(mod, seed=33, std=0.05, perturb_layer_norm=True)
    x_q, x_k, mask_q, mask_k, logits, scq, sck = _cross_inputs(s, 34)
    ref = oracle.cross_attention(x_q, x_k, mask_q, mask_k, logits, _params(mod), scq, sck, 4)
    mod = mod.to(DEV)
    args = [t.to(DEV) for t in (x_q, x_k, mask_q, mask_k, logits, scq, sck)]
    with torch.inference_mode():
        upd = mod(*args)
        assert upd.shape == (s, NQ, C) and upd.dtype == torch.bfloat16
        assert oracle.relative_error(upd.float().cpu(), ref) < TOL
        acc = args[0].clone()
        mod.accumulate_(acc, args[1], *args[2:])
    assert oracle.relative_error(acc.cpu() - x_q, ref) < TOL


def test_cross_attention_masked_rows_average_masked_keys():
    """The reference's 1e9 * !mask_q * !mask_k term: a masked query attends
    uniformly to the masked keys of its window (the logits differ by far less
    than the spacing of floats near 1e9), whatever its own logits."""
    s = 2
    mod = CrossAttention().eval()
    init_params_(mod, seed=35, std=0.05)
    x_q, x_k, mask_q, mask_k, logits, scq, sck = _cross_inputs(s, 36)
    mask_q[1, :] = False
    ref = oracle.cross_attention(x_q, x_k, mask_q, mask_k, logits, _params(mod), scq, sck, 4)
    mod = mod.to(DEV)
    with torch.inference_mode():
        upd = mod(*(t.to(DEV) for t in (x_q, x_k, mask_q, mask_k, logits, scq, sck)))
    assert oracle.relative_error(upd[1].float().cpu(), ref[1]) < TOL


def test_cross_attention_key_gather_is_exact():
    """The gather fused into the keys' LayerNorm reads the same rows as
    atom_layout.convert: bit-identical updates."""
    s = 7
    info, qmask, kmask = windows(s, 21)
    mod = CrossAttention().eval()
    init_params_(mod, seed=37, std=0.05, perturb_layer_norm=True)
    g = torch.Generator().manual_seed(38)
    x_q = torch.randn(s, NQ, C, generator=g)
    logits = torch.randn(s, 4, NQ, NK, generator=g)
    scq = torch.randn(s, NQ, C, generator=g)
    mod = mod.to(DEV)
    with torch.inference_mode():
        xq, scq_d = x_q.to(DEV), scq.to(DEV)
        sck = atom_layout.convert(info, scq_d, layout_axes=(-3, -2))
        x_k = atom_layout.convert(info, xq, layout_axes=(-3, -2))
        keys = atom_layout.key_gather(info, s * NQ, DEV)
        a = mod._run(xq, keys, qmask.to(DEV), kmask.to(DEV), logits.to(DEV), scq_d, sck, None, False)
        b = mod(xq, x_k, qmask.to(DEV), kmask.to(DEV), logits.to(DEV), scq_d, sck)
    assert torch.equal(a, b)


def test_cross_attention_gather_index_out_of_range_reads_zeros():
    """An index outside the source rows (passed straight to the library) is
    caught by the LayerNorm kernel's own bounds check: the row reads zeros, as
    an invalid gather entry does, and device error 0x106 is set."""
    s = 2
    info, qmask, kmask = windows(s, 0)
    mod = CrossAttention().eval()
    init_params_(mod, seed=39, std=0.05).to(DEV)
    g = torch.Generator().manual_seed(40)
    x_q = torch.randn(s, NQ, C, generator=g).to(DEV)
    with torch.inference_mode():
        idx, valid = atom_layout.key_gather(info, s * NQ, DEV)
        bad_idx = idx.clone()
        assert bool(valid[1, 20])  # key 20 of subset 1 is row 4 of the atoms
        bad_idx[1, 20] = s * NQ  # one past the last row
        zero_valid = valid.clone()
        zero_valid[1, 20] = False
        sc = torch.randn(s, NQ, C, generator=g).to(DEV)
        sck = atom_layout.convert(info, sc, layout_axes=(-3, -2))
        ref = mod._run(x_q, (idx, zero_valid), None, None, None, sc, sck, None, False)
        torch.cuda.synchronize()
        assert _capi.device_error(clear=True) == 0
        got = mod._run(x_q, (bad_idx, valid), None, None, None, sc, sck, None, False)
        torch.cuda.synchronize()
        assert _capi.device_error(clear=True) == 0x106
    assert torch.equal(got, ref)


@pytest.mark.parametrize("subsets,tail", [(8, 19), (3, 0)])
def test_diffusion_cross_att_transformer(subsets, tail):
    mod = DiffusionCrossAttTransformer().eval()
    init_params_(mod, seed=41, std=0.05, perturb_layer_norm=True)
    info, qmask, kmask = windows(subsets, tail)
    g = torch.Generator().manual_seed(42)
    act = torch.randn(subsets, NQ, C, generator=g)
    qsc = torch.randn(subsets, NQ, C, generator=g)
    ksc = oracle.atom_layout_convert(info.gather_idxs, info.gather_mask, qsc)
    pair_cond = torch.randn(subsets, NQ, NK, 16, generator=g)
    ref = oracle.diffusion_cross_att_transformer(act, qmask, info.gather_idxs, info.gather_mask,
                                                 kmask, qsc, ksc, pair_cond, _params(mod))
    mod = mod.to(DEV)
    a = act.to(DEV)
    with torch.inference_mode():
        out = mod(a, qmask.to(DEV), info, kmask.to(DEV), qsc.to(DEV), ksc.to(DEV), pair_cond.to(DEV))
    assert out is a
    assert oracle.relative_error(a.cpu() - act, ref - act) < TOL


def test_cross_attention_rejects_other_widths():
    mod = CrossAttention(key_dim=64, value_dim=64, c_single_cond=64, num_head=4).to(DEV)
    x = torch.randn(1, NQ, 64, device=DEV)
    with pytest.raises(ValueError):
        mod(x, torch.randn(1, NK, 64, device=DEV), torch.ones(1, NQ, device=DEV),
            torch.ones(1, NK, device=DEV), None, torch.randn(1, NQ, 64, device=DEV),
            torch.randn(1, NK, 64, device=DEV))


def test_cross_att_transformer_cuda_graph_matches_eager():
    """A captured atom transformer replays the same kernels: bit-identical to
    the eager blocks on inputs that were not the ones captured."""
    s = 6
    mod = DiffusionCrossAttTransformer().eval()
    init_params_(mod, seed=43, std=0.05, perturb_layer_norm=True)
    info, qmask, kmask = windows(s, 9)
    g = torch.Generator().manual_seed(44)
    act = torch.randn(s, NQ, C, generator=g)
    qsc = torch.randn(s, NQ, C, generator=g)
    pair_cond = torch.randn(s, NQ, NK, 16, generator=g)
    mod = mod.to(DEV)
    with torch.inference_mode():
        qsc_d = qsc.to(DEV)
        ksc_d = atom_layout.convert(info, qsc_d, layout_axes=(-3, -2))
        args = (qmask.to(DEV), info, kmask.to(DEV))
        step = mod.capture(act.to(DEV), *args, qsc_d, ksc_d, pair_cond.to(DEV))
        for k in range(2):
            a2 = torch.randn(s, NQ, C, generator=g).to(DEV)
            q2 = torch.randn(s, NQ, C, generator=g).to(DEV)
            k2 = atom_layout.convert(info, q2, layout_axes=(-3, -2))
            got = step(a2, q2, k2).clone()
            want = a2.clone()
            mod(want, *args, q2, k2, pair_cond.to(DEV))
            torch.cuda.synchronize()
            assert torch.equal(got, want), k
