"""The reference's own modules and bridges, driven into this library through
its af3_kernels-compatible ABI (xfold_cpu_b200.af3_compat, xfb_af3_* entry
points).

The reference is imported from baseline/_ref (installed unmodified by
`pip install --no-deps --target baseline/_ref` of the reference checkout).  Its
`cpp` backend reaches native code through two functions of
xfold/fastnn/native.py: `load_native_operator` (:7-18), which returns
`af3_kernels._C`, and `check_cpu_inference` (:21-28), which refuses
non-CPU tensors.  The tests replace exactly those two -- the extension with
af3_compat, the device check with one that accepts CUDA tensors, which is the
whole of the integration a maintainer adds -- and run the reference's own
forward methods (`TriangleMultiplication._forward_cpp`,
`GridSelfAttention` with `linear_cpp` and `dot_product_attention_cpp`,
`SelfAttention._forward_cpp`, `PairformerBlock.forward`) on CUDA tensors.
The comparison is the same module instance on its `torch` backend, on the
same GPU in float32; the bar is the bf16 one, max |got - ref| / max |ref| <=
1e-2 on the updates.
"""

import sys
from contextlib import contextmanager
from pathlib import Path

import pytest
import torch

import oracle
from xfold_cpu_b200 import _capi, af3_compat

pytestmark = pytest.mark.gpu

REF_DIR = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
TOL = 1e-2
DEV = "cuda"


@pytest.fixture(scope="module")
def xfold():
    if not (REF_DIR / "xfold").is_dir():
        pytest.skip("the reference is not installed in baseline/_ref")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import xfold.fastnn.config as config
    import xfold.fastnn.native as native
    import xfold.nn.attention as attention
    import xfold.nn.diffusion_transformer as diffusion_transformer
    import xfold.nn.pairformer as pairformer
    import xfold.nn.primitives as primitives
    import xfold.nn.triangle_multiplication as triangle_multiplication
    return {"config": config, "native": native, "attention": attention,
            "pairformer": pairformer, "primitives": primitives,
            "triangle_multiplication": triangle_multiplication,
            "diffusion_transformer": diffusion_transformer}


def _check_cuda_inference(*tensors):
    """The reference's check_cpu_inference with CUDA tensors accepted."""
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda or t.layout != torch.strided:
            raise ValueError("Native operators require strided CUDA tensors.")
        if torch.is_grad_enabled() and t.requires_grad:
            raise RuntimeError("Native operators support inference only; disable gradients.")


@contextmanager
def backend(xfold, name):
    """Selects the reference's `torch` backend, or its `cpp` backend wired to af3_compat."""
    cfg, nat = xfold["config"], xfold["native"]
    saved = (cfg.triangle_multiplication_implementation, cfg.dot_product_attention_implementation,
             nat.load_native_operator, nat.check_cpu_inference)
    try:
        cfg.triangle_multiplication_implementation = name
        cfg.dot_product_attention_implementation = name
        if name == "cpp":
            nat.load_native_operator = lambda op: af3_compat.load_extension()
            nat.check_cpu_inference = _check_cuda_inference
        yield
    finally:
        (cfg.triangle_multiplication_implementation, cfg.dot_product_attention_implementation,
         nat.load_native_operator, nat.check_cpu_inference) = saved


def _init(module, seed):
    """Weights ~ N(0, 0.02), LayerNorm gamma ~ 1 + 0.1 N, beta ~ 0.1 N (CPU generator)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            leaf = name.rsplit(".", 1)[-1]
            owner = module.get_submodule(name.rsplit(".", 1)[0]) if "." in name else module
            if type(owner).__name__ == "LayerNorm":
                v = torch.randn(p.shape, generator=g) * 0.1
                p.copy_(v + 1.0 if leaf == "weight" else v)
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    return module.to(DEV).eval()


def _pair(n, seed, tail):
    g = torch.Generator().manual_seed(seed)
    pair = torch.randn(n, n, 128, generator=g)
    m = torch.ones(n)
    m[n - tail:] = 0
    return pair.to(DEV), (m[:, None] * m[None, :]).to(DEV), m.to(DEV)


def _rel(got, ref):
    return oracle.relative_error(got.float().cpu(), ref.float().cpu())


@pytest.fixture(autouse=True)
def _no_device_error():
    _capi.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert _capi.device_error(clear=True) == 0


@pytest.mark.parametrize("outgoing", [True, False], ids=["outgoing", "incoming"])
def test_reference_triangle_multiplication_cpp_bridge(xfold, outgoing):
    mod = _init(xfold["triangle_multiplication"].TriangleMultiplication(128, _outgoing=outgoing), 1)
    pair, mask, _ = _pair(96, 2, 6)
    with torch.inference_mode():
        with backend(xfold, "torch"):
            ref = mod(pair, mask)
        with backend(xfold, "cpp"):
            got = mod(pair, mask)
    assert got.dtype == ref.dtype and got.shape == ref.shape
    assert _rel(got, ref) < TOL


@pytest.mark.parametrize("transpose", [False, True], ids=["starting", "ending"])
def test_reference_grid_self_attention_cpp_bridge(xfold, transpose):
    """linear_cpp for the bias, q / k / v, gate and output projections (the
    4-wide bias included) and dot_product_attention_cpp for the attention."""
    mod = _init(xfold["attention"].GridSelfAttention(128, 4, transpose=transpose), 3)
    pair, mask, _ = _pair(80, 4, 8)
    with torch.inference_mode():
        with backend(xfold, "torch"):
            ref = mod(pair, mask)
        with backend(xfold, "cpp"):
            got = mod(pair, mask)
    assert _rel(got, ref) < TOL


def test_reference_single_attention_cpp_bridge(xfold):
    """SelfAttention._forward_cpp (q bias, 16 heads of 24, pair logits, 1-D mask)."""
    mod = _init(xfold["diffusion_transformer"].SelfAttention(c_x=384, num_head=16,
                                                             use_single_cond=False), 5)
    g = torch.Generator().manual_seed(6)
    n = 72
    x = torch.randn(n, 384, generator=g).to(DEV)
    logits = torch.randn(16, n, n, generator=g).to(DEV)
    mask = torch.ones(n, device=DEV)
    mask[-5:] = 0
    with torch.inference_mode():
        with backend(xfold, "torch"):
            ref = mod(x, mask, pair_logits=logits)
        with backend(xfold, "cpp"):
            got = mod(x, mask, pair_logits=logits)
    assert _rel(got, ref) < TOL


def test_reference_pairformer_block_cpp_backend(xfold):
    """A whole reference PairformerBlock with its triangle and attention
    switches on `cpp`, i.e. on this library, against the same block on torch."""
    blk = _init(xfold["pairformer"].PairformerBlock(), 7)
    pair, mask, seq = _pair(64, 8, 4)
    single = torch.randn(64, 384, generator=torch.Generator().manual_seed(9)).to(DEV)
    with torch.inference_mode():
        with backend(xfold, "torch"):
            ref_pair, ref_single = blk(pair.clone(), mask, single.clone(), seq)
        with backend(xfold, "cpp"):
            got_pair, got_single = blk(pair.clone(), mask, single.clone(), seq)
    assert _rel(got_pair - pair, ref_pair - pair) < TOL
    assert _rel(got_single - single, ref_single - single) < TOL


def test_reference_gated_linear_unit_and_linear_abi(xfold):
    """The raw af3 functions against the reference's torch formulas: GLU with
    the transposed weight [K, 2N] (gated_linear_unit_torch,
    xfold/fastnn/gated_linear_unit.py:103-107) and linear with [K, N] plus bias
    (native.py:55-70), output widths 4 (padded) and 256."""
    import importlib

    # xfold.fastnn re-exports a function of the same name as this submodule
    glu = importlib.import_module("xfold.fastnn.gated_linear_unit")

    g = torch.Generator().manual_seed(11)
    x = torch.randn(3, 50, 128, generator=g).to(DEV)
    w = (torch.randn(128, 2 * 512, generator=g) * 0.05).to(DEV)
    with torch.inference_mode():
        got = af3_compat.gated_linear_unit(x, w, M_BLK=64, N_BLK=32)
        ref = glu.gated_linear_unit_torch(x, w)
        assert got.shape == ref.shape and got.dtype == ref.dtype
        assert _rel(got, ref) < TOL
        for n in (4, 256):
            wl = (torch.randn(128, n, generator=g) * 0.05).to(DEV)
            b = torch.randn(n, generator=g).to(DEV)
            got = af3_compat.linear(x, wl, b)
            assert got.shape == (3, 50, n)
            assert _rel(got, x @ wl + b) < TOL
        with pytest.raises(RuntimeError, match="positive LIBXSMM"):
            af3_compat.gated_linear_unit(x, w, M_BLK=0)
        with pytest.raises(RuntimeError, match="VNNI2"):
            af3_compat.linear(x, w, weight_packed=True)
