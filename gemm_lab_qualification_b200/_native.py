"""ctypes binding of libglq.so, the C ABI declared in include/glq.h.

This module is the only place Python touches the native library.  It loads
the in-tree ``libglq.so`` (built by ``gemm_lab_qualification_b200.build``)
and fails loudly when it is missing: there is no Python or torch fallback for
any compute call.  Device memory, streams and dtypes come from torch tensors;
only raw pointers, element strides and sizes cross the boundary.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libglq.so"

# enum glq_dtype / glq_epilogue / glq_path / glq_status (include/glq.h)
DTYPE_F16, DTYPE_BF16 = 0, 1
EPILOGUE_NONE, EPILOGUE_BIAS, EPILOGUE_BIAS_SILU = 0, 1, 2
PATHS = ("empty", "zero_k", "gemv_m1", "tc_tcgen05", "tc_splitk", "tail", "strided", "unaligned", "tc_kn",
         "repacked", "tc_ldg")
STATUS_OK = 0
STATUS_NAMES = ("ok", "invalid_argument", "shape", "split", "workspace", "output_layout", "cuda",
                "device", "device_timeout", "scratch")
MAX_SPLIT = 8
MAX_RANKS = 8
STATIC_GATHER_SLOTS = 64
FLAG_NO_PDL = 1 << 0
FLAG_STATIC_WEIGHTS = 1 << 1

# Every symbol include/glq.h declares, with (restype, argtypes).
_I64 = ctypes.c_int64
_VP = ctypes.c_void_p
_INT = ctypes.c_int
_PINT = ctypes.POINTER(ctypes.c_int)
SIGNATURES = {
    "glq_linear": (_INT, [_INT, _VP, _I64, _I64, _VP, _I64, _I64, _VP, _INT, _VP, _I64, _I64, _I64,
                          _I64, _INT, _VP, ctypes.c_size_t, _VP, _PINT, _PINT]),
    "glq_linear_ex": (_INT, [_INT, _VP, _I64, _I64, _VP, _I64, _I64, _VP, _INT, _VP, _I64, _I64, _I64,
                             _I64, _INT, _VP, ctypes.c_size_t, _VP, ctypes.c_uint, _PINT, _PINT]),
    "glq_linear_f16": (_INT, [_VP, _I64, _I64, _VP, _I64, _I64, _VP, _VP, _I64, _INT, _INT, _INT,
                              _INT, _VP, ctypes.c_size_t, _VP, _PINT]),
    "glq_matmul": (_INT, [_INT, _VP, _VP, _VP, _INT, _INT, _INT, _VP]),
    "glq_splitk_matmul": (_INT, [_INT, _VP, _VP, _VP, _INT, _INT, _INT, _VP, _INT, _VP]),
    "glq_linear_gather": (_INT, [_INT, _VP, _I64, _I64, _VP, _I64, _I64, _VP, _INT, ctypes.POINTER(_VP), _I64,
                                 _I64, _I64, _I64, _I64, _INT, _INT, _INT, ctypes.POINTER(_VP),
                                 ctypes.POINTER(ctypes.c_uint), ctypes.c_uint64, _VP, ctypes.c_uint, _PINT, _PINT]),
    "glq_linear_gather_static": (_INT, [_INT, _VP, _I64, _I64, _VP, _I64, _I64, _VP, _INT, ctypes.POINTER(_VP),
                                        _I64, _I64, _I64, _I64, _I64, _INT, _INT, _INT, ctypes.POINTER(_VP),
                                        _INT, ctypes.c_uint64, _VP, ctypes.c_uint, _PINT, _PINT]),
    "glq_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64, _INT]),
    "glq_linear_workspace_bytes": (ctypes.c_size_t, [_INT, _VP, _I64, _I64, _VP, _I64, _I64, _I64, _I64, _I64]),
    "glq_plan": (_INT, [_INT, _VP, _I64, _I64, _VP, _I64, _I64, _I64, _I64, _I64, _I64, _INT, _INT,
                        _PINT, _PINT]),
    "glq_path_name": (ctypes.c_char_p, [_INT]),
    "glq_status_string": (ctypes.c_char_p, [_INT]),
    "glq_device_error": (_INT, [ctypes.POINTER(ctypes.c_uint), _INT]),
    "glq_abi_version": (_INT, []),
    "glq_build_target": (ctypes.c_char_p, []),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeLibraryMissing(ImportError):
    """libglq.so is not built; the operators have no other implementation."""


class GlqError(RuntimeError):
    """A libglq.so call returned a non-OK glq_status."""

    def __init__(self, status: int, what: str):
        self.status = status
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"{what}: glq status {status} ({name}): {status_string(status)}")


def library() -> ctypes.CDLL:
    """Load libglq.so once; raise NativeLibraryMissing if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIBRARY_PATH.exists():
                raise NativeLibraryMissing(
                    f"{LIBRARY_PATH} is missing; build it with "
                    "`python -m gemm_lab_qualification_b200.build` (nvcc, sm_100a)")
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    return library().glq_status_string(status).decode()


def path_name(path: int) -> str:
    return library().glq_path_name(path).decode()


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return DTYPE_F16
    if dtype == torch.bfloat16:
        return DTYPE_BF16
    raise ValueError("inputs must share dtype float16 or bfloat16")


def workspace_bytes(m: int, n: int, k: int, split_k: int = 0) -> int:
    return int(library().glq_workspace_bytes(m, n, k, split_k))


def linear_workspace_bytes(dtype: int, a_ptr: int, a_strides: tuple[int, int], b_ptr: int,
                           b_strides: tuple[int, int], m: int, n: int, k: int) -> int:
    """Workspace with which glq_linear copies strided or unaligned operands
    into aligned rows and runs the tcgen05 / GEMV kernel (0: not needed)."""
    return int(library().glq_linear_workspace_bytes(dtype, a_ptr, a_strides[0], a_strides[1], b_ptr, b_strides[0],
                                                    b_strides[1], m, n, k))


def plan(dtype: int, a_ptr: int, a_strides: tuple[int, int], b_ptr: int, b_strides: tuple[int, int],
         y_row_stride: int, m: int, n: int, k: int, split_k: int = 0, sm_count: int = 0) -> tuple[str, int]:
    """Path name and split a call would take (pure host query, no launch)."""
    path = ctypes.c_int(-1)
    split = ctypes.c_int(0)
    status = library().glq_plan(dtype, a_ptr, a_strides[0], a_strides[1], b_ptr, b_strides[0],
                                b_strides[1], y_row_stride, m, n, k, split_k, sm_count,
                                ctypes.byref(path), ctypes.byref(split))
    if status != STATUS_OK:
        raise GlqError(status, "glq_plan")
    return PATHS[path.value], split.value


def linear(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, bias: torch.Tensor | None = None,
           epilogue: int = EPILOGUE_NONE, split_k: int = 0, workspace: torch.Tensor | None = None,
           stream: torch.cuda.Stream | None = None, flags: int = 0) -> tuple[str, int]:
    """out = epilogue(a @ b [+ bias]) through glq_linear on the current stream.

    a: [M, K], b: [K, N] (any strides; W[N, K].T is the K-contiguous fast
    layout), out: [M, N] with unit column stride.  Returns (path, split).
    """
    m, k = a.shape
    n = b.shape[1]
    if stream is None:
        stream = torch.cuda.current_stream(out.device) if out.is_cuda else None
    handle = stream.cuda_stream if stream is not None else 0
    ws_ptr = workspace.data_ptr() if workspace is not None else None
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    path = ctypes.c_int(-1)
    split = ctypes.c_int(0)
    status = library().glq_linear_ex(
        dtype_code(a.dtype),
        a.data_ptr(), a.stride(0), a.stride(1),
        b.data_ptr(), b.stride(0), b.stride(1),
        bias.data_ptr() if bias is not None else None, epilogue,
        out.data_ptr(), out.stride(0),
        m, n, k, split_k, ws_ptr, ws_bytes, handle, flags,
        ctypes.byref(path), ctypes.byref(split))
    if status != STATUS_OK:
        raise GlqError(status, "glq_linear_ex")
    return PATHS[path.value], split.value


def linear_gather(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None, epilogue: int,
                  y_ptrs: list[int], y_row_stride: int, y_col_offset: int, rank: int,
                  signal_ptrs: list[int], counter_ptr: int, epoch: int, split_k: int = 0,
                  stream: torch.cuda.Stream | None = None, flags: int = 0) -> tuple[str, int]:
    """One rank's column-parallel linear with the all-gather fused in (glq_linear_gather).

    y_ptrs / signal_ptrs: per rank, device pointers mapped in this process to
    that rank's output buffer and signal slots; this rank's N columns land at
    y_col_offset in every rank's buffer.  Returns (path, split).
    """
    m, k = a.shape
    n = b.shape[1]
    world = len(y_ptrs)
    if stream is None:
        stream = torch.cuda.current_stream(a.device)
    ys = (_VP * world)(*y_ptrs)
    sigs = (_VP * world)(*signal_ptrs)
    path = ctypes.c_int(-1)
    split = ctypes.c_int(0)
    status = library().glq_linear_gather(
        dtype_code(a.dtype),
        a.data_ptr(), a.stride(0), a.stride(1),
        b.data_ptr(), b.stride(0), b.stride(1),
        bias.data_ptr() if bias is not None else None, epilogue,
        ys, y_row_stride, y_col_offset, m, n, k, split_k, rank, world,
        sigs, ctypes.cast(ctypes.c_void_p(counter_ptr), ctypes.POINTER(ctypes.c_uint)), epoch,
        stream.cuda_stream, flags, ctypes.byref(path), ctypes.byref(split))
    if status != STATUS_OK:
        raise GlqError(status, "glq_linear_gather")
    return PATHS[path.value], split.value


def device_error(clear: bool = True) -> int:
    """Sticky in-kernel error word of the current device (0 = none)."""
    word = ctypes.c_uint(0)
    status = library().glq_device_error(ctypes.byref(word), 1 if clear else 0)
    if status != STATUS_OK:
        raise GlqError(status, "glq_device_error")
    return int(word.value)
