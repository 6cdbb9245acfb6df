"""The C-ABI library loads and exports every function include/xfold_b200.h
declares (no device work: this runs without a GPU)."""

import re
from pathlib import Path

import pytest

from xfold_cpu_b200 import _capi
from xfold_cpu_b200.build import LIB_PATH

HEADER = Path(__file__).resolve().parents[1] / "include" / "xfold_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"XFB_API\s+[\w\s\*]+?\b(xfb_\w+)\s*\(", text)))


def test_header_declares_the_operator_set():
    names = declared_symbols()
    for required in ("xfb_triangle_multiplication", "xfb_dot_product_attention",
                     "xfb_gated_linear_unit", "xfb_linear", "xfb_layer_norm", "xfb_runtime_info",
                     "xfb_gemm", "xfb_grid_self_attention", "xfb_transition", "xfb_self_attention"):
        assert required in names


@pytest.mark.skipif(not LIB_PATH.exists(), reason="library not built")
def test_library_exports_every_declared_symbol():
    lib = _capi.load()
    missing = [name for name in declared_symbols() if not hasattr(lib, name)]
    assert not missing, missing


def test_binding_table_matches_header():
    assert sorted(_capi.SIGNATURES) == declared_symbols()


@pytest.mark.skipif(not LIB_PATH.exists(), reason="library not built")
def test_workspace_queries_need_no_device():
    lib = _capi.load()
    assert lib.xfb_triangle_multiplication_workspace(1024, 128) > 4 * 1024 * 1024 * 128
    assert lib.xfb_grid_self_attention_workspace(64, 128, 4) > 0
    assert lib.xfb_transition_workspace(100, 128, 4) > 0


@pytest.mark.skipif(not LIB_PATH.exists(), reason="library not built")
def test_argument_errors_are_reported_without_a_device():
    lib = _capi.load()
    rc = lib.xfb_linear(None, 4, 7, None, 8, None, None, 0, 0, None)
    assert rc == _capi.ERR_INVALID
    assert "multiples of 8" in _capi.last_error()


def _c_layout(struct: str, fields: list[str]) -> list[int]:
    """sizeof and offsetof of a header struct, from a C program compiled with gcc."""
    import shutil
    import subprocess
    import tempfile

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    body = "".join(f'  printf("%zu\\n", offsetof({struct}, {f}));\n' for f in fields)
    src = ('#include <stdio.h>\n#include <stddef.h>\n'
           f'#include "{HEADER}"\nint main(void) {{\n'
           f'  printf("%zu\\n", sizeof({struct}));\n{body}  return 0;\n}}\n')
    with tempfile.TemporaryDirectory() as tmp:
        c, exe = Path(tmp) / "layout.c", Path(tmp) / "layout"
        c.write_text(src)
        subprocess.run(["gcc", "-o", str(exe), str(c)], check=True, capture_output=True)
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return [int(v) for v in out.split()]


@pytest.mark.parametrize("cls,struct", [(_capi.F32GemmArgs, "xfb_f32_gemm_args"),
                                        (_capi.F32AttentionArgs, "xfb_f32_attention_args"),
                                        (_capi.CopyBox, "xfb_copy_box")])
def test_ctypes_structs_match_header_layout(cls, struct):
    names = [name for name, _ in cls._fields_]
    got = [ctypes_sizeof(cls)] + [getattr(cls, n).offset for n in names]
    assert got == _c_layout(struct, names)


def ctypes_sizeof(cls) -> int:
    import ctypes

    return ctypes.sizeof(cls)


@pytest.mark.skipif(not LIB_PATH.exists(), reason="library not built")
def test_new_entry_points_reject_bad_arguments_without_a_device():
    """Argument checks of the routed stages, the float32 path and the checkpoint
    scatter run before any device work."""
    import ctypes

    lib = _capi.load()
    p = ctypes.c_void_p
    dst = (p * 2)(16, 32)
    # routed contraction: rank outside the world
    assert lib.xfb_triangle_contraction_routed(None, None, 4, 64, 1, dst, 2, 5, None) == \
        _capi.ERR_INVALID
    assert "rank" in _capi.last_error()
    # routed destinations must be non-null
    null_dst = (p * 2)(16, None)
    assert lib.xfb_grid_attention_prepare_routed(None, 0, 32, 64, 128, 4, None, None, 1e-5, None,
                                                 null_dst, 2, 0, None, None) == _capi.ERR_INVALID
    # float32 GEMM: unknown activation
    args = _capi.F32GemmArgs()
    args.m = args.n = args.k = args.batch = 4
    args.act = 2
    assert lib.xfb_f32_gemm(ctypes.addressof(args), None) == _capi.ERR_INVALID
    # float32 LayerNorm wider than 1024 columns
    assert lib.xfb_f32_layer_norm(None, 4, 2048, 2048, None, None, 1e-5, None, 2048, None) == \
        _capi.ERR_INVALID
    # checkpoint scatter: a span past the end of the source blob
    spans = (ctypes.c_int64 * 3)(100, 0, 64)
    assert lib.xfb_gather_bytes(16, 128, 32, 1024, spans, spans, 1, None) == _capi.ERR_INVALID
    assert "outside the source" in _capi.last_error()
