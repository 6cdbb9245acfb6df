"""The allocation-free GLU entry point, checked through the C ABI.

xfb_gated_linear_unit_noalloc serves callers that cannot give this library
device memory (a host runtime that owns every allocation through its own pool,
or a service whose footprint must stay fixed after start-up): it keeps its
scratch in a fixed array inside the library instead of a caller workspace.
Its output must agree with xfb_gated_linear_unit (which packs the weight into
a caller workspace) within the tolerance of the other GPU tests, on two calls
in a row with different shapes, so the second call cannot lean on what the
first left in the shared scratch.

This file is named to be collected last: it runs after every other test, and
also passes alone in a fresh process.
"""

import pytest
import torch

import oracle
from xfold_cpu_b200 import _capi

pytestmark = pytest.mark.gpu

TOL = 1e-2
MAX_WEIGHT_ELEMS = 4 * 1024 * 1024  # XFB_GLU_NOALLOC_MAX_WEIGHT_ELEMS in include/xfold_b200.h


def _glu_workspace(x, w, n):
    """The existing entry point, with a workspace from torch's allocator."""
    lib = _capi.load()
    m, k = x.shape
    y = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    ws_bytes = lib.xfb_gated_linear_unit_workspace(m, k, n)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    _capi.check(lib.xfb_gated_linear_unit(x.data_ptr(), m, k, w.data_ptr(), n, 0, y.data_ptr(),
                                          ws.data_ptr(), ws_bytes,
                                          torch.cuda.current_stream().cuda_stream),
                "xfb_gated_linear_unit")
    return y


def _glu_noalloc(x, w, n):
    lib = _capi.load()
    m, k = x.shape
    y = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    _capi.check(lib.xfb_gated_linear_unit_noalloc(x.data_ptr(), m, k, w.data_ptr(), n,
                                                  y.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream),
                "xfb_gated_linear_unit_noalloc")
    return y


def test_noalloc_glu_matches_the_workspace_entry_point_on_two_calls():
    _capi.device_error(clear=True)
    g = torch.Generator(device="cuda").manual_seed(5)
    # second call: a larger weight than the first, so stale scratch would show
    for m, k, n in ((777, 128, 512), (300, 384, 1536)):
        x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
        w = (torch.randn(2 * n, k, device="cuda", generator=g) * 0.1).bfloat16()
        ref = _glu_workspace(x, w, n)
        got = _glu_noalloc(x, w, n)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert oracle.relative_error(got.float().cpu(), ref.float().cpu()) <= TOL
    assert _capi.device_error(clear=True) == 0


def test_noalloc_glu_matches_the_oracle_at_the_scratch_limit_and_on_empty_input():
    """Checked against the CPU oracle on its own (not only against the
    workspace entry point, which shares the packing and GEMM kernels), with a
    weight that fills the scratch exactly (2 n k = the maximum) followed by a
    call with no rows."""
    _capi.device_error(clear=True)
    g = torch.Generator(device="cuda").manual_seed(6)
    m, k, n = 260, 1024, 2048
    assert 2 * n * k == MAX_WEIGHT_ELEMS
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(2 * n, k, device="cuda", generator=g) * 0.05).bfloat16()
    got = _glu_noalloc(x, w, n)
    torch.cuda.synchronize()
    ref = oracle.gated_linear_unit(x.float().cpu(), w.float().cpu().T)
    assert oracle.relative_error(got.float().cpu(), ref) <= TOL
    empty = _glu_noalloc(torch.zeros(0, k, dtype=torch.bfloat16, device="cuda"), w, n)
    torch.cuda.synchronize()
    assert empty.shape == (0, n)
    assert _capi.device_error(clear=True) == 0


def test_noalloc_glu_rejects_weights_beyond_the_scratch():
    x = torch.zeros(128, 1024, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(2 * 4096, 1024, dtype=torch.bfloat16, device="cuda")  # 8M elements
    with pytest.raises(ValueError, match="exceeds the fixed scratch"):
        _glu_noalloc(x, w, 4096)
    # sizes whose product 2 n k would overflow 64 bits are rejected by the same check
    lib = _capi.load()
    rc = lib.xfb_gated_linear_unit_noalloc(x.data_ptr(), 128, 1 << 40, w.data_ptr(), 1 << 40,
                                           x.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # XFB_ERR_INVALID
