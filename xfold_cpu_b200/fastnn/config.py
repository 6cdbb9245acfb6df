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
