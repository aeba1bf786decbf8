"""B200 (sm_100a) rebuild of the GEMM lab's FP16 linear (+ bias + SiLU) path.

* ``kernels`` -- the lab's operator API (``triton_matmul``,
  ``triton_bias_silu``, ``triton_splitk_matmul``, the Plans, the
  ``gemm_lab::*`` custom ops) backed by the native kernels.
* ``_native`` -- ctypes binding of ``libglq.so`` (C ABI in include/glq.h).
* ``workloads`` -- the qualification contract's deterministic inputs.
* ``evidence`` -- CUDA-event timing and statistics of the lab's harness.
* ``build`` -- the nvcc recipe for ``libglq.so`` and ``gemm_bench``.

The Python package name uses underscores because a Python package cannot
contain hyphens.
"""
from __future__ import annotations

__version__ = "0.1.0"


def library_path() -> str:
    from ._native import LIBRARY_PATH
    return str(LIBRARY_PATH)
