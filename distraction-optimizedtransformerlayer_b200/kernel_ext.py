"""Loader for libdotl, the sm_100a kernel library behind `optimized/`.

Drop-in for the reference's kernel_ext.py (kernel_ext.py:363-491 upstream):
`get_kernels()` returns the module of tensor-level entry points (same names
and arguments as the reference's pybind module `transformer_kernels`), or None
with the reason in `load_error()` when the library cannot be loaded.

The difference is how the library is made. The reference JIT-builds a pybind
extension for whatever GPU is present. This one is a plain C-ABI shared
library (include/dotl.h) compiled ahead of time for sm_100a, in-tree, by
`build()`; `get_kernels()` only builds when the library file is missing.
The tensor-level functions bind it through ctypes in `dotl_ops.py`.
"""

from __future__ import annotations

import os
import subprocess
from typing import List, Optional

_THIS_DIR = os.path.dirname(os.path.abspath(__file__))
_CSRC = os.path.join(_THIS_DIR, "csrc")
_LIB_DIR = os.path.join(_THIS_DIR, "lib")
LIB_PATH = os.path.join(_LIB_DIR, "libdotl.so")
HEADER_PATH = os.path.join(os.path.dirname(_THIS_DIR), "include", "dotl.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    # Share the process's libcudart (torch loads libcudart.so.12), so the
    # current device set by torch is the one these entry points see.
    "-cudart", "shared",
]

_kernels = None
_load_attempted = False
_load_error: Optional[BaseException] = None


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(home, "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def build_command() -> List[str]:
    return [_nvcc(), *NVCC_FLAGS, "-o", LIB_PATH, os.path.join(_CSRC, "dotl.cu")]


def build(verbose: bool = False) -> str:
    """Compile csrc/dotl.cu into lib/libdotl.so for sm_100a. Returns the path.

    Cross-compiles without a GPU. Raises RuntimeError with nvcc's output on
    failure.
    """
    os.makedirs(_LIB_DIR, exist_ok=True)
    cmd = build_command()
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or proc.returncode != 0:
        print(" ".join(cmd))
        print(proc.stdout + proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr[-4000:]}")
    return LIB_PATH


def get_kernels(verbose: bool = False):
    """The tensor-level kernel module (dotl_ops), or None if unavailable.

    None means the library could not be loaded or CUDA is absent; the reason
    is in load_error(). Callers that have no alternative path (all of
    `optimized/`) raise on None rather than substituting anything.
    """
    global _kernels, _load_attempted, _load_error
    if _load_attempted:
        return _kernels
    _load_attempted = True
    try:
        import torch

        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is not available")
        if not os.path.exists(LIB_PATH):
            build(verbose)
        import dotl_ops

        dotl_ops.load(LIB_PATH)
        _kernels = dotl_ops
    except BaseException as exc:  # noqa: BLE001 - reported through load_error()
        _kernels = None
        _load_error = exc
    return _kernels


def load_error() -> Optional[BaseException]:
    """Whatever went wrong during the last get_kernels() attempt, if anything."""
    return _load_error
