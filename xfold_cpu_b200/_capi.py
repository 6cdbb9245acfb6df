"""ctypes binding of libxfold_b200.so (include/xfold_b200.h).

The library is loaded on first use.  A missing library, a missing symbol or a
non-sm_100 device raises RuntimeError / ValueError: there is no fallback path.
"""

from __future__ import annotations

import ctypes
import json
import threading
from pathlib import Path

from .build import LIB_PATH

F32, BF16, U8 = 0, 1, 2
OK, ERR_INVALID, ERR_CUDA, ERR_DEVICE, ERR_TIMEOUT = 0, 1, 2, 3, 4

_i = ctypes.c_int
_i64 = ctypes.c_int64
_u32p = ctypes.POINTER(ctypes.c_uint32)
_p = ctypes.c_void_p
_d = ctypes.c_double
_s = ctypes.c_char_p

# name -> (restype, argtypes), in header order.
SIGNATURES: dict[str, tuple] = {
    "xfb_last_error": (_s, []),
    "xfb_launch_count": (ctypes.c_uint64, []),
    "xfb_runtime_info": (_i, [_s, _i64]),
    "xfb_check_device": (_i, []),
    "xfb_device_error": (_i, [_i, _u32p]),
    "xfb_selftest_wait_timeout": (_i, [_i64, _p]),
    "xfb_layer_norm": (_i, [_p, _i, _i64, _i64, _p, _p, _d, _p, _p]),
    "xfb_linear": (_i, [_p, _i64, _i64, _p, _i64, _p, _p, _i, _i, _p]),
    "xfb_gemm": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i, _i, _i, _p]),
    "xfb_pack_glu_weight_bytes": (_i64, [_i64, _i64]),
    "xfb_pack_glu_weight": (_i, [_p, _i, _i64, _i64, _p, _p]),
    "xfb_gated_linear_unit_workspace": (_i64, [_i64, _i64, _i64]),
    "xfb_gated_linear_unit": (_i, [_p, _i64, _i64, _p, _i64, _i, _p, _p, _i64, _p]),
    "xfb_gated_linear_unit_noalloc": (_i, [_p, _i64, _i64, _p, _i64, _p, _p]),
    "xfb_pack_triangle_weights_bytes": (_i64, [_i64]),
    "xfb_pack_triangle_weights": (_i, [_p, _p, _p, _i, _i64, _p, _p]),
    "xfb_triangle_multiplication_workspace": (_i64, [_i64, _i64]),
    "xfb_triangle_multiplication": (
        _i,
        [_p, _i, _i64, _i64, _p, _i, _p, _p, _p, _p, _p, _p, _p, _p, _d, _d, _i, _p, _p, _i,
         _i, _p, _i64, _p],
    ),
    "xfb_dot_product_attention_workspace": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "xfb_dot_product_attention": (
        _i,
        [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i, _i, _p, _i, _i, _i, _p, _p, _i64,
         _p],
    ),
    "xfb_pack_attention_weights_bytes": (_i64, [_i64]),
    "xfb_pack_attention_weights": (_i, [_p, _p, _p, _p, _i, _i64, _p, _p]),
    "xfb_grid_self_attention_workspace": (_i64, [_i64, _i64, _i64]),
    "xfb_grid_self_attention": (
        _i,
        [_p, _i, _i64, _i64, _i64, _p, _i, _p, _p, _d, _p, _p, _p, _p, _p, _p, _i, _p, _p, _i,
         _i, _p, _i64, _p],
    ),
    "xfb_transition_workspace": (_i64, [_i64, _i64, _i64]),
    "xfb_transition": (
        _i,
        [_p, _i, _i64, _i64, _i64, _p, _p, _d, _p, _p, _p, _i, _p, _p, _p, _i, _i, _p, _i64,
         _p],
    ),
    "xfb_self_attention_workspace": (_i64, [_i64, _i64, _i64]),
    "xfb_self_attention": (
        _i,
        [_p, _i, _i64, _i64, _i64, _p, _p, _p, _p, _d, _p, _p, _p, _p, _p, _p, _p, _i, _p, _p,
         _p, _p, _i, _i, _p, _i64, _p],
    ),
    "xfb_pair_logits": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _d, _p, _p, _p]),
    # row-block stages of the row-sharded pair
    "xfb_triangle_projection_workspace": (_i64, [_i64, _i64, _i64]),
    "xfb_triangle_projection": (
        _i, [_p, _i, _i64, _i64, _i64, _p, _p, _p, _d, _p, _p, _p, _p, _p, _i64, _p]),
    "xfb_triangle_output_workspace": (_i64, [_i64, _i64, _i64]),
    "xfb_triangle_output": (
        _i, [_p, _i64, _i64, _i64, _p, _p, _p, _d, _p, _p, _i, _i, _p, _i64, _p]),
    "xfb_grid_attention_prepare": (
        _i, [_p, _i, _i64, _i64, _i64, _i64, _p, _p, _d, _p, _p, _p, _p]),
    "xfb_grid_attention_rows_workspace": (_i64, [_i64, _i64, _i64, _i64]),
    "xfb_grid_attention_rows": (
        _i, [_p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i, _i, _p, _i64, _p]),
    "xfb_grid_attention_core_workspace": (_i64, [_i64, _i64]),
    "xfb_grid_attention_core": (_i, [_p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _p]),
    "xfb_pair_logits_rows": (_i, [_p, _i, _i64, _i64, _i64, _i64, _p, _p, _d, _p, _p, _p]),
    "xfb_triangle_projection_routed": (
        _i, [_p, _i, _i64, _i64, _i64, _p, _p, _p, _d, _p, _p, _p, _i, _i, _p, _p, _i64, _p]),
    "xfb_triangle_contraction_routed": (_i, [_p, _p, _i64, _i64, _i, _p, _i, _i, _p]),
    "xfb_grid_attention_prepare_routed": (
        _i, [_p, _i, _i64, _i64, _i64, _i64, _p, _p, _d, _p, _p, _i, _i, _p, _p]),
    "xfb_grid_attention_rows_routed": (
        _i, [_p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i, _i, _p, _i64, _p]),
    "xfb_self_attention_rows_workspace": (_i64, [_i64, _i64, _i64, _i64]),
    "xfb_self_attention_rows": (
        _i, [_p, _i, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _d, _p, _p, _p, _p, _p, _i,
             _i, _p, _i64, _p]),
    "xfb_exchange_copy": (_i, [_p, _i, _p]),
    "xfb_ipc_handle_bytes": (_i64, []),
    "xfb_ipc_handle": (_i, [_p, _p, ctypes.POINTER(ctypes.c_int64)]),
    "xfb_ipc_open": (_i, [_p, _i64, ctypes.POINTER(ctypes.c_void_p)]),
    "xfb_ipc_close": (_i, [_p, _i64]),
    "xfb_exchange_signal": (_i, [_p, _i, _i, ctypes.c_uint32, _p]),
    "xfb_exchange_wait": (_i, [_p, _i, ctypes.c_uint32, _p]),
    "xfb_exchange_signal_counted": (_i, [_p, _i, _i, _p, _p]),
    "xfb_exchange_wait_counted": (_i, [_p, _i, _p, _p]),
    "xfb_conditioning": (_i, [_p, _i64, _i64, _p, _i64, _p, _i64, _i, _p, _p]),
    "xfb_cross_pair_logits": (_i, [_p, _i, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _d, _p,
                                   _p, _p]),
    "xfb_cross_attention_workspace": (_i64, [_i64]),
    "xfb_msa_attention_workspace": (_i64, [_i64, _i64]),
    "xfb_pack_outer_product_weight_bytes": (_i64, [_i64]),
    "xfb_pack_outer_product_weight": (_i, [_p, _i, _i64, _p, _p]),
    "xfb_outer_product_mean_workspace": (_i64, [_i64, _i64]),
    "xfb_outer_product_mean": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _p, _d, _p, _p, _p, _p,
                                    _i64, _p, _i, _p, _i64, _p]),
    "xfb_msa_attention": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _i, _i64, _i64, _p, _p, _p, _p,
                               _d, _p, _p, _p, _p, _p, _i, _i, _p, _i64, _p]),
    "xfb_cross_attention": (_i, [_p, _i, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _p,
                                 _p, _d, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _p, _i64,
                                 _p]),
    "xfb_af3_linear_workspace": (_i64, [_i64, _i64]),
    "xfb_af3_linear": (_i, [_p, _i64, _i64, _p, _i, _i64, _p, _i, _p, _i, _p, _i64, _p]),
    "xfb_af3_gated_linear_unit_workspace": (_i64, [_i64, _i64]),
    "xfb_af3_gated_linear_unit": (
        _i, [_p, _i64, _i64, _p, _i, _i64, _i64, _i64, _i, _p, _p, _i64, _p]),
    "xfb_af3_triangle_multiplication_workspace": (_i64, [_i64, _i64]),
    "xfb_af3_triangle_multiplication": (
        _i,
        [_p, _i, _i64, _i64, _p, _i, _p, _p, _p, _p, _p, _p, _p, _p, _i, _d, _d, _i64, _i, _p,
         _i, _p, _i64, _p],
    ),
    "xfb_af3_dot_product_attention_workspace": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "xfb_af3_dot_product_attention": (
        _i,
        [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i, _i, _p, _i, _i, _i64, _i, _p, _p,
         _i64, _p],
    ),
    "xfb_f32_gemm": (_i, [_p, _p]),
    "xfb_f32_layer_norm": (_i, [_p, _i64, _i64, _i64, _p, _p, _d, _p, _i64, _p]),
    "xfb_f32_attention": (_i, [_p, _p]),
    "xfb_f32_silu_mul": (_i, [_p, _i64, _i64, _p, _p]),
    "xfb_f32_scale_shift": (_i, [_p, _p, _p, _i64, _p]),
    "xfb_gather_bytes": (_i, [_p, _i64, _p, _i64, _p, _p, _i64, _p]),
}


def _fields(spec: str) -> list:
    """ctypes fields from 'name:type ...' (p = pointer, l = int64, i = int, d = double)."""
    kinds = {"p": ctypes.c_void_p, "l": ctypes.c_int64, "i": ctypes.c_int, "d": ctypes.c_double}
    return [(name, kinds[t]) for name, t in (f.split(":") for f in spec.split())]


class F32GemmArgs(ctypes.Structure):
    """xfb_f32_gemm_args (include/xfold_b200.h)."""

    _fields_ = _fields("a:p a_sb:l a_si:l a_sk:l b:p b_sb:l b_sj:l b_sk:l c:p c_sb:l c_si:l "
                       "c_sj:l m:l n:l k:l batch:l bias:p act:i row_scale:p rs_sb:l rs_si:l "
                       "mul:p mul_sb:l mul_si:l mul_sj:l accumulate:i")


class F32AttentionArgs(ctypes.Structure):
    """xfb_f32_attention_args (include/xfold_b200.h)."""

    _fields_ = _fields("q:p q_sb:l q_sh:l q_si:l k:p k_sb:l k_sh:l k_si:l v:p v_sb:l v_sh:l "
                       "v_si:l bias:p bias_sb:l bias_sh:l bias_si:l mask:p mask_sb:l out:p "
                       "out_sb:l out_sh:l out_si:l gate:p gate_sb:l gate_sh:l gate_si:l batch:l "
                       "heads:l nq:l nk:l d:l dv:l scale:d")


class CopyBox(ctypes.Structure):
    """xfb_copy_box (include/xfold_b200.h)."""

    _fields_ = [("src", ctypes.c_void_p), ("dst", ctypes.c_void_p), ("d0", ctypes.c_int64),
                ("d1", ctypes.c_int64), ("d2_bytes", ctypes.c_int64),
                ("src_stride0", ctypes.c_int64), ("src_stride1", ctypes.c_int64),
                ("dst_stride0", ctypes.c_int64), ("dst_stride1", ctypes.c_int64)]

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Loads the shared library and declares every exported function."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -c 'import __graft_entry__ as g; "
                "g.build()'` or xfold_cpu_b200.build.build_library()"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError as error:
                raise RuntimeError(f"{LIB_PATH.name} does not export {name}; rebuild it") from error
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def last_error() -> str:
    return load().xfb_last_error().decode("utf-8", "replace")


def check(rc: int, what: str) -> None:
    """Raises the Python error that matches a C-ABI status code."""
    if rc == OK:
        return
    message = f"{what}: {last_error()}"
    if rc == ERR_INVALID:
        raise ValueError(message)
    raise RuntimeError(message)


def call(name: str, *args):
    fn = getattr(load(), name)
    rc = fn(*args)
    check(rc, name)
    return rc


def runtime_info() -> dict:
    buf = ctypes.create_string_buffer(1024)
    call("xfb_runtime_info", buf, len(buf))
    return json.loads(buf.value.decode())


def launch_count() -> int:
    """Kernels launched by the library in this process."""
    return int(load().xfb_launch_count())


def device_error(clear: bool = True) -> int:
    code = ctypes.c_uint32(0)
    call("xfb_device_error", 1 if clear else 0, ctypes.byref(code))
    return int(code.value)
