"""Operator backend switch, mirroring xfold/fastnn/config.py:2-16.

The reference selects per-op implementations from module globals read at
every forward call ("torch", "triton", "cpp", "ipex").  This package adds the
"cuda" implementation (hand-written sm_100a kernels behind a C ABI) and
implements only that one: any other value raises ValueError at the call, as
the reference does for unknown names, and an explicit selection never falls
back silently (the reference's contract, tests/test_glu_static.py:60-69).
"""

CUDA = "cuda"
SUPPORTED = (CUDA,)

# Arithmetic of the `cuda` modules: "bfloat16" (tensor cores, the reference's
# autocast route) or "float32" (CUDA-core fp32 kernels, the reference's
# no-autocast route, matched to 1e-4).
BFLOAT16, FLOAT32 = "bfloat16", "float32"
compute_dtype = BFLOAT16

layer_norm_implementation = CUDA
dot_product_attention_implementation = CUDA
gated_linear_unit_implementation = CUDA
triangle_multiplication_implementation = CUDA


def require_cuda(option_name: str) -> None:
    value = globals()[option_name]
    if value != CUDA:
        raise ValueError(
            f"{option_name}={value!r}: xfold_cpu_b200 implements only the 'cuda' backend; "
            "use xfold's own modules for 'torch' / 'triton' / 'cpp' / 'ipex'"
        )


def float32() -> bool:
    """True when the modules compute in float32 (compute_dtype)."""
    if compute_dtype not in (BFLOAT16, FLOAT32):
        raise ValueError(f"compute_dtype={compute_dtype!r}: expected 'bfloat16' or 'float32'")
    return compute_dtype == FLOAT32
