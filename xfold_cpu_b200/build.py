"""Builds libxfold_b200.so (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

The library is a single translation unit (csrc/capi.cu) that includes every
kernel header.  It links the CUDA runtime statically, so it depends only on
the NVIDIA driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
LIB_NAME = "libxfold_b200.so"
LIB_PATH = PACKAGE_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
BASE_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-shared",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-cudart",
    "static",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [
        PACKAGE_DIR.parent / "include" / "xfold_b200.h"
    ]


def needs_rebuild() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def build_library(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compiles csrc/capi.cu into xfold_cpu_b200/libxfold_b200.so (sm_100a)."""
    if not force and not needs_rebuild():
        return LIB_PATH
    flags = ARCH_FLAGS + BASE_FLAGS + list(extra_flags or [])
    flag_text = " ".join(ARCH_FLAGS + ["-O3", "-lineinfo"])
    cmd = [nvcc_path(), *flags, f'-DXFB_NVCC_FLAGS="{flag_text}"', str(CSRC / "capi.cu"),
           "-o", str(LIB_PATH) + ".tmp"]
    if verbose:
        print(" ".join(cmd))
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(result.stdout, result.stderr)
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    build_library(force="--force" in sys.argv, verbose=True,
                  extra_flags=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None)
    print(LIB_PATH)
