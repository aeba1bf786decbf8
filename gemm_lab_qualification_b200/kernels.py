"""Operator API of the GEMM lab, backed by the sm_100a kernels of libglq.so.

Drop-in for the reference module ``kernels.py``: the same public names,
argument meanings, output allocation rules and ``ValueError`` contract
violations, with every Triton body replaced by one call through the C ABI
(``include/glq.h``).  Differences, each deliberate:

* Inputs need not be contiguous.  The reference rejects any non-contiguous
  operand (kernels.py:143-144), which also rejects ``W.T``, the layout of a
  linear layer's weight.  Here ``b = W.T`` (strides ``(1, K)``) is the
  primary fast layout, the reference's contiguous ``b = [K, N]`` is accepted
  as well, and strided / misaligned views each take an explicit GPU path.
* There is one native path per call and no vendor or torch fallback: the
  ``adaptive_*`` names keep their signatures but always run the native
  kernels; the ``*_path`` helpers report the native path name.
* Every call records the GPU path it took; ``last_path()`` returns it.
* ``launch_options(pdl=..., static_weights=...)`` sets per-thread launch
  flags: programmatic dependent launch (on by default; stream semantics
  unchanged) and the opt-in declaration that the weight operand is not
  written by the preceding kernel, which lets a call start streaming it
  before its predecessor finishes.

Cited reference lines are in ``kernels.py`` of the reference project.
"""
from __future__ import annotations

import threading

import torch

from . import _native

__all__ = [
    "triton_matmul_into", "triton_matmul", "TritonMatmulPlan",
    "triton_bias_silu_into", "triton_bias_silu", "TritonBiasSiluPlan",
    "adaptive_bias_silu_path", "adaptive_bias_silu",
    "triton_splitk_matmul_into", "triton_splitk_matmul", "TritonSplitKPlan",
    "AdaptiveMatmulPlan", "TritonAdaptivePlan", "adaptive_path", "triton_adaptive_matmul",
    "linear_into", "last_path", "planned_path", "launch_options",
]

_last = threading.local()
_options = threading.local()


class launch_options:
    """Per-thread launch flags for the native calls made inside the block.

    pdl: launch with programmatic dependent launch (default True).
    static_weights: the ``b`` operand is not written by the kernel that
    precedes each call in its stream (inference weights); the kernels then
    request it before waiting for that kernel (default False).
    """

    def __init__(self, pdl: bool = True, static_weights: bool = False) -> None:
        self.flags = (0 if pdl else _native.FLAG_NO_PDL) | (_native.FLAG_STATIC_WEIGHTS if static_weights else 0)
        self._saved = 0

    def __enter__(self) -> "launch_options":
        self._saved = getattr(_options, "flags", 0)
        _options.flags = self.flags
        return self

    def __exit__(self, *exc) -> None:
        _options.flags = self._saved


def _flags() -> int:
    return getattr(_options, "flags", 0)


def last_path() -> tuple[str, int] | None:
    """(path, split) of the most recent native call made by this thread."""
    return getattr(_last, "value", None)


def _record(result: tuple[str, int]) -> None:
    _last.value = result


_ext = None


def _binding():
    """The native call path (csrc/glq_torch.cpp): argument checks with the
    messages below plus the glq_linear_ex launch, in one C++ call."""
    global _ext
    if _ext is None:
        _native.library()  # fails loudly when libglq.so is missing
        try:
            from . import _glq_torch
        except ImportError as exc:
            raise _native.NativeLibraryMissing(
                "the _glq_torch binding is not built; build it with "
                "`python -m gemm_lab_qualification_b200.build`") from exc
        _ext = _glq_torch
    return _ext


def _launch(op: str, a: torch.Tensor, b: torch.Tensor, output: torch.Tensor, bias: torch.Tensor | None = None,
            epilogue: int = _native.EPILOGUE_NONE, split_k: int = 0, partial: torch.Tensor | None = None) -> None:
    status, path, split = _binding().linear(op, a, b, output, bias, epilogue, split_k, partial, _flags())
    if status != _native.STATUS_OK:
        raise _native.GlqError(status, "glq_linear_ex")
    _last.value = (_native.PATHS[path], split)


def _validate_inputs(a: torch.Tensor, b: torch.Tensor, operation: str) -> tuple[int, int, int]:
    """Contract checks of kernels.py:132-145, minus the contiguity rule."""
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError(f"{operation} expects two rank-2 tensors")
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"incompatible dimensions: {tuple(a.shape)} and {tuple(b.shape)}")
    if a.device.type != "cuda" or b.device.type != "cuda":
        raise ValueError(f"{operation} requires CUDA tensors")
    if a.device != b.device:
        raise ValueError("input tensors must be on the same CUDA device")
    if a.dtype != b.dtype or a.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("inputs must share dtype float16 or bfloat16")
    return int(a.shape[0]), int(b.shape[1]), int(a.shape[1])


def _validate_output(output: torch.Tensor, a: torch.Tensor, m: int, n: int) -> None:
    if tuple(output.shape) != (m, n) or output.device != a.device or output.dtype != a.dtype:
        raise ValueError("output tensor has the wrong shape, device, or dtype")
    # Row-major rows, possibly padded: unit column stride, row stride >= n.
    if m and n and ((n > 1 and output.stride(1) != 1) or (m > 1 and output.stride(0) < n)):
        raise ValueError("output tensor must be contiguous")


def _validate_bias(bias: torch.Tensor, a: torch.Tensor, n: int) -> None:
    if bias.ndim != 1 or bias.shape[0] != n or bias.device != a.device or bias.dtype != a.dtype:
        raise ValueError("bias tensor has the wrong shape, device, or dtype")
    if n > 1 and bias.stride(0) != 1:
        raise ValueError("bias tensor must be contiguous")


def linear_into(a: torch.Tensor, b: torch.Tensor, output: torch.Tensor, bias: torch.Tensor | None = None,
                activation: str | None = None, split_k: int = 0,
                partial: torch.Tensor | None = None) -> torch.Tensor:
    """General form: output = act(a @ b [+ bias]); act in {None, 'silu'}."""
    if activation not in (None, "silu"):
        raise ValueError("activation must be None or 'silu'")
    if activation == "silu" and bias is None:
        raise ValueError("the fused SiLU epilogue takes a bias")
    epilogue = (_native.EPILOGUE_NONE if bias is None else
                _native.EPILOGUE_BIAS_SILU if activation == "silu" else _native.EPILOGUE_BIAS)
    _launch("linear", a, b, output, bias, epilogue, split_k, partial)
    return output


def planned_path(a: torch.Tensor, b: torch.Tensor, split_k: int = 0) -> tuple[str, int]:
    """(path, split) a call on these tensors would take; no launch."""
    m, k = a.shape
    n = b.shape[1]
    return _native.plan(_native.dtype_code(a.dtype), a.data_ptr(), tuple(a.stride()), b.data_ptr(),
                        tuple(b.stride()), n, m, n, k, split_k)


# ---------------------------------------------------------------- GEMM (kernels.py:148-188)

def triton_matmul_into(a: torch.Tensor, b: torch.Tensor, output: torch.Tensor) -> torch.Tensor:
    _launch("triton_matmul", a, b, output)
    return output


def triton_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    m, n, _ = _validate_inputs(a, b, "triton_matmul")
    output = torch.empty((m, n), device=a.device, dtype=a.dtype)
    return triton_matmul_into(a, b, output)


class TritonMatmulPlan:
    def __init__(self, a: torch.Tensor, b: torch.Tensor) -> None:
        m, n, _ = _validate_inputs(a, b, "triton_matmul")
        self.a = a
        self.b = b
        self.output = torch.empty((m, n), device=a.device, dtype=a.dtype)

    def __call__(self) -> torch.Tensor:
        return triton_matmul_into(self.a, self.b, self.output)


# ---------------------------------------------------------------- bias + SiLU (kernels.py:252-321)

def triton_bias_silu_into(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor,
                          output: torch.Tensor) -> torch.Tensor:
    _launch("triton_bias_silu", a, b, output, bias, _native.EPILOGUE_BIAS_SILU)
    return output


def triton_bias_silu(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    m, n, _ = _validate_inputs(a, b, "triton_bias_silu")
    output = torch.empty((m, n), device=a.device, dtype=a.dtype)
    return triton_bias_silu_into(a, b, bias, output)


def adaptive_bias_silu_path(m: int, n: int, k: int, dtype: torch.dtype | None = None) -> str:
    """Native path of a fused call on contiguous A and a K-contiguous W.

    The reference gates a Triton path on two MLP shapes (kernels.py:289-298);
    here every shape runs the native fused kernel.
    """
    code = _native.dtype_code(dtype if dtype is not None else torch.float16)
    return _native.plan(code, 0, (k, 1), 0, (1, k), n, m, n, k)[0]


def adaptive_bias_silu(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    _validate_inputs(a, b, "adaptive_bias_silu")
    return triton_bias_silu(a, b, bias)


class TritonBiasSiluPlan:
    def __init__(self, a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> None:
        m, n, _ = _validate_inputs(a, b, "triton_bias_silu")
        self.a = a
        self.b = b
        self.bias = bias
        self.output = torch.empty((m, n), device=a.device, dtype=a.dtype)

    def __call__(self) -> torch.Tensor:
        return triton_bias_silu_into(self.a, self.b, self.bias, self.output)


# ---------------------------------------------------------------- split-K (kernels.py:396-470)

def triton_splitk_matmul_into(a: torch.Tensor, b: torch.Tensor, partial: torch.Tensor,
                              output: torch.Tensor, split_k: int = 4) -> torch.Tensor:
    """Forced split-K: per-split FP32 sums land in ``partial`` ([S, M, N]) and
    are merged in-kernel in split order (no second launch)."""
    if split_k not in (2, 4, 8):
        raise ValueError("split_k must be 2, 4, or 8")
    m, n, _ = _validate_inputs(a, b, "triton_splitk_matmul")
    if tuple(partial.shape) != (split_k, m, n) or partial.device != a.device or partial.dtype != torch.float32:
        raise ValueError("partial tensor has the wrong shape, device, or dtype")
    if not partial.is_contiguous():
        raise ValueError("partial tensor must be contiguous")
    _launch("triton_splitk_matmul", a, b, output, None, _native.EPILOGUE_NONE, split_k, partial)
    return output


def triton_splitk_matmul(a: torch.Tensor, b: torch.Tensor, split_k: int = 4) -> torch.Tensor:
    m, n, _ = _validate_inputs(a, b, "triton_splitk_matmul")
    partial = torch.empty((split_k, m, n), device=a.device, dtype=torch.float32)
    output = torch.empty((m, n), device=a.device, dtype=a.dtype)
    return triton_splitk_matmul_into(a, b, partial, output, split_k)


class TritonSplitKPlan:
    def __init__(self, a: torch.Tensor, b: torch.Tensor, split_k: int = 4) -> None:
        if split_k not in (2, 4, 8):
            raise ValueError("split_k must be 2, 4, or 8")
        m, n, _ = _validate_inputs(a, b, "triton_splitk_matmul")
        self.a = a
        self.b = b
        self.split_k = split_k
        self.partial = torch.empty((split_k, m, n), device=a.device, dtype=torch.float32)
        self.output = torch.empty((m, n), device=a.device, dtype=a.dtype)

    def workspace_bytes(self) -> int:
        """FP32 partial-sum storage held outside the output tensor."""
        return self.partial.numel() * self.partial.element_size()

    def __call__(self) -> torch.Tensor:
        return triton_splitk_matmul_into(self.a, self.b, self.partial, self.output, self.split_k)


# ---------------------------------------------------------------- adaptive (kernels.py:473-513)

def adaptive_path(m: int, n: int, k: int, dtype: torch.dtype | None = None) -> str:
    """Native path for contiguous A and K-contiguous W (kernels.py:493-499)."""
    code = _native.dtype_code(dtype if dtype is not None else torch.float16)
    return _native.plan(code, 0, (k, 1), 0, (1, k), n, m, n, k)[0]


class AdaptiveMatmulPlan:
    def __init__(self, a: torch.Tensor, b: torch.Tensor) -> None:
        m, n, k = _validate_inputs(a, b, "triton_adaptive_matmul")
        self.selected_path = planned_path(a, b)[0]
        self.plan = TritonMatmulPlan(a, b)

    def workspace_bytes(self) -> int:
        """The native merge needs no workspace."""
        return 0

    def __call__(self) -> torch.Tensor:
        return self.plan()


def triton_adaptive_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("incompatible rank-2 matrix shapes")
    return triton_matmul(a, b)


# Backward-compatible name (kernels.py:513).
TritonAdaptivePlan = AdaptiveMatmulPlan


# ---------------------------------------------------------------- torch custom ops (kernels.py:516-617)

def _fake_mm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("incompatible matrix shapes")
    return torch.empty((a.shape[0], b.shape[1]), device=a.device, dtype=a.dtype)


def _fake_bias_silu(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    if a.ndim != 2 or b.ndim != 2 or bias.ndim != 1 or a.shape[1] != b.shape[0]:
        raise ValueError("incompatible matrix/bias shapes")
    if b.shape[1] != bias.shape[0]:
        raise ValueError("bias length must match output columns")
    return torch.empty((a.shape[0], b.shape[1]), device=a.device, dtype=a.dtype)


@torch.library.custom_op("gemm_lab::triton_matmul", mutates_args=())
def triton_matmul_op(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Inference custom op backed by the native sm_100a kernels."""
    return triton_matmul(a, b)


triton_matmul_op.register_fake(_fake_mm)


@torch.library.custom_op("gemm_lab::triton_splitk_matmul", mutates_args=())
def triton_splitk_matmul_op(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Split-K (S = 4) custom op with the in-kernel merge."""
    return triton_splitk_matmul(a, b, split_k=4)


triton_splitk_matmul_op.register_fake(_fake_mm)


@torch.library.custom_op("gemm_lab::triton_adaptive_matmul", mutates_args=())
def triton_adaptive_matmul_op(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Adaptive custom op: the library's own split choice."""
    return triton_adaptive_matmul(a, b)


triton_adaptive_matmul_op.register_fake(_fake_mm)


@torch.library.custom_op("gemm_lab::adaptive_matmul", mutates_args=())
def adaptive_matmul_op(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Same native path as gemm_lab::triton_adaptive_matmul."""
    return triton_adaptive_matmul(a, b)


adaptive_matmul_op.register_fake(_fake_mm)


@torch.library.custom_op("gemm_lab::triton_bias_silu", mutates_args=())
def triton_bias_silu_op(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """Fused inference epilogue: output = SiLU(A @ B + bias)."""
    return triton_bias_silu(a, b, bias)


triton_bias_silu_op.register_fake(_fake_bias_silu)


@torch.library.custom_op("gemm_lab::adaptive_bias_silu", mutates_args=())
def adaptive_bias_silu_op(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """Fused epilogue; every shape takes the native fused kernel."""
    return adaptive_bias_silu(a, b, bias)


adaptive_bias_silu_op.register_fake(_fake_bias_silu)
