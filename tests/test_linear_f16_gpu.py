"""glq_linear_f16, the reference-facing C entry point, called directly.

This is the one-call FP16 form a foreign host binds (cgo / JNI / ctypes):
A with a row stride and a column stride, B given by its row and column
strides (B = W^T as strides (1, K) for a linear layer's K-contiguous weight,
or the lab's own contiguous B = [K, N] as (N, 1)), an optional bias, and Y
with a row stride.  A non-null bias selects the fused epilogue
SiLU(A B + bias); a null bias the plain product A B.  Checked against the
CPU FP64 oracle on the seed-7 uniform sweep at the uniform gate
abs <= 0.02 + 0.002 * |ref| (kernels.py:252-286 and qualification.py:24-56 of
the reference are the contract).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gemm_lab_qualification_b200 import _native as native
from gemm_lab_qualification_b200 import workloads
from oracle import reference as oracle

pytestmark = pytest.mark.gpu

U_ATOL, U_RTOL = oracle.UNIFORM_ATOL, oracle.UNIFORM_RTOL


@pytest.fixture(autouse=True)
def clean_error_word(cuda_device):
    native.device_error(clear=True)
    yield
    assert native.device_error(clear=True) == 0, "a bounded in-kernel wait expired"


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def call_f16(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None, y: torch.Tensor) -> str:
    """glq_linear_f16 on torch's current stream, no workspace; returns the path name."""
    lib = native.library()
    m, k = a.shape
    n = b.shape[1]
    path = ctypes.c_int(-1)
    status = lib.glq_linear_f16(a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0), b.stride(1),
                                bias.data_ptr() if bias is not None else None, y.data_ptr(), y.stride(0), m, n, k,
                                0, None, 0, torch.cuda.current_stream().cuda_stream, ctypes.byref(path))
    assert status == native.STATUS_OK, native.status_string(status)
    return native.PATHS[path.value]


@pytest.mark.parametrize("layout", ["w_t", "b_kn"])
@pytest.mark.parametrize("with_bias", [True, False])
@pytest.mark.parametrize("m", [1, 8, 32, 128])
def test_linear_f16_sweep(cuda_device, m, with_bias, layout):
    a, w, bias = workloads.uniform_inputs(m, 4096, 4096)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    b = dw.t() if layout == "w_t" else dw.t().contiguous()
    assert b.stride() == ((1, 4096) if layout == "w_t" else (4096, 1))
    y = torch.full((m, 4096), 123, dtype=torch.float16, device=cuda_device)
    path = call_f16(da, b, db if with_bias else None, y)
    assert path not in ("empty", "zero_k", "strided", "unaligned")
    torch.cuda.synchronize()
    expected = oracle.linear_reference(a, w, bias if with_bias else None, silu=with_bias)
    oracle.compare(host(y), expected, U_ATOL, U_RTOL)


def test_linear_f16_matches_operator_api_bitwise(cuda_device):
    """Same inputs through glq_linear_f16 and the operator API: same bits."""
    from gemm_lab_qualification_b200 import kernels
    a, w, bias = workloads.uniform_inputs(32, 4096, 4096)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    y = torch.empty((32, 4096), dtype=torch.float16, device=cuda_device)
    call_f16(da, dw.t(), db, y)
    ref = kernels.triton_bias_silu(da, dw.t(), db)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


def test_linear_f16_odd_pointer_refused(cuda_device):
    """An odd element address is refused before any launch."""
    lib = native.library()
    a, w, bias = workloads.uniform_inputs(8, 512, 512)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    y = torch.empty((8, 512), dtype=torch.float16, device=cuda_device)
    status = lib.glq_linear_f16(da.data_ptr(), 512, 1, dw.data_ptr(), 1, 512, db.data_ptr() + 1, y.data_ptr(),
                                512, 8, 512, 512, 0, None, 0, torch.cuda.current_stream().cuda_stream, None)
    assert native.STATUS_NAMES[status] == "invalid_argument"
