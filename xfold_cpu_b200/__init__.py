"""B200-native (sm_100a) Pairformer / diffusion hot path for xfold.

The CUDA kernels live in libxfold_b200.so (C ABI, include/xfold_b200.h),
loaded through ctypes by `_capi`.  `native` holds the torch-tensor wrappers
that mirror af3_kernels._C; `fastnn` and `nn` mirror xfold's operator switch
and modules with a `cuda` backend.
"""

__version__ = "0.1.0"
