"""glq_linear_gather_static: the fused gather for callers that cannot allocate.

Some callers of the column-parallel layer only hold device pointers handed
to them (weights, activations, the communicator's peer-mapped output and
signal buffers) and have no allocator of their own, so they cannot supply
the private arrival counter that glq_linear_gather needs.  The static entry
point takes that counter from an array compiled into the library.  This test
drives it through the C ABI on one GPU (one rank, its own signal slots) and
checks that two calls in a row give the same output as the allocating entry
point and the FP64 oracle's gate.

The file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
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
ERR_TIMEOUT_PEER = 1 << 5


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def call_static(a, w, bias, out, sig, slot, epoch):
    """One rank of one: output and signal slots are this test's own buffers."""
    lib = native.library()
    ys = (ctypes.c_void_p * 1)(out.data_ptr())
    sigs = (ctypes.c_void_p * 1)(sig.data_ptr())
    path, split = ctypes.c_int(-1), ctypes.c_int(0)
    m, k = a.shape
    n = w.shape[0]
    status = lib.glq_linear_gather_static(
        native.DTYPE_F16, a.data_ptr(), a.stride(0), 1, w.data_ptr(), 1, w.stride(0), bias.data_ptr(),
        native.EPILOGUE_BIAS_SILU, ys, out.stride(0), 0, m, n, k, 0, 0, 1, sigs, slot, epoch,
        torch.cuda.current_stream().cuda_stream, 0, ctypes.byref(path), ctypes.byref(split))
    return status, native.PATHS[path.value] if path.value >= 0 else None


@pytest.mark.parametrize("m", [32, 1])
def test_static_gather_matches_allocating_entry_point(cuda_device, m):
    native.device_error(clear=True)
    a, w, bias = workloads.uniform_inputs(m, 4096, 4096)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    expected = oracle.linear_reference(a, w, bias, silu=True)

    # the allocating entry point, with a counter this test allocated
    ref = torch.empty((m, 4096), dtype=torch.float16, device=cuda_device)
    ref_sig = torch.zeros(native.MAX_RANKS, dtype=torch.int64, device=cuda_device)
    counter = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    native.linear_gather(da, dw.t(), db, native.EPILOGUE_BIAS_SILU, [ref.data_ptr()], 4096, 0, 0,
                         [ref_sig.data_ptr()], counter.data_ptr(), 1)

    # two calls in a row through the static scratch (the first and last slots)
    sig = torch.zeros(native.MAX_RANKS, dtype=torch.int64, device=cuda_device)
    for epoch, slot in ((1, 0), (2, native.STATIC_GATHER_SLOTS - 1)):
        out = torch.full((m, 4096), 123, dtype=torch.float16, device=cuda_device)
        status, path = call_static(da, dw, db, out, sig, slot, epoch)
        assert status == 0, native.status_string(status)
        torch.cuda.synchronize()
        oracle.compare(host(out), expected, U_ATOL, U_RTOL)
        # the same kernel on the same inputs: the same bits
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        assert int(sig[0]) == epoch
    assert native.device_error(clear=True) == 0


def test_static_gather_slot_reused_after_an_expired_wait(cuda_device):
    """A slot whose last call ended in an expired wait serves the next call.

    Each call clears its slot on the stream before the launch, so whatever an
    interrupted call left there does not leak into the next one.  One launch,
    one GPU: the emulated second rank's signal slot is never written, so the
    kernel's bounded peer wait (about 1 s) runs out, the kernel returns and
    reports it in the device error word; then a one-rank call with a later
    epoch on the same slot completes and matches the oracle."""
    native.device_error(clear=True)
    m, n, k = 8, 1024, 1024
    a, w, bias = workloads.uniform_inputs(m, n, k)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    expected = oracle.linear_reference(a, w, bias, silu=True)
    lib = native.library()
    slot = 5
    outs = [torch.zeros((m, 2 * n), dtype=torch.float16, device=cuda_device) for _ in range(2)]
    sigs = [torch.zeros(native.MAX_RANKS, dtype=torch.int64, device=cuda_device) for _ in range(2)]
    ys = (ctypes.c_void_p * 2)(*[o.data_ptr() for o in outs])
    sp = (ctypes.c_void_p * 2)(*[s.data_ptr() for s in sigs])
    path, split = ctypes.c_int(-1), ctypes.c_int(0)
    status = lib.glq_linear_gather_static(
        native.DTYPE_F16, da.data_ptr(), k, 1, dw.data_ptr(), 1, k, db.data_ptr(), native.EPILOGUE_BIAS_SILU, ys,
        2 * n, 0, m, n, k, 0, 0, 2, sp, slot, 3, torch.cuda.current_stream().cuda_stream, 0, ctypes.byref(path),
        ctypes.byref(split))
    assert status == 0, native.status_string(status)
    torch.cuda.synchronize()
    assert native.device_error(clear=True) & ERR_TIMEOUT_PEER
    assert native.device_error(clear=True) == 0
    # the same slot, a one-rank call with a later epoch
    out = torch.full((m, n), 123, dtype=torch.float16, device=cuda_device)
    sig = torch.zeros(native.MAX_RANKS, dtype=torch.int64, device=cuda_device)
    status, _ = call_static(da, dw, db, out, sig, slot, 4)
    assert status == 0, native.status_string(status)
    torch.cuda.synchronize()
    oracle.compare(host(out), expected, U_ATOL, U_RTOL)
    assert int(sig[0]) == 4
    assert native.device_error(clear=True) == 0


def test_static_gather_refuses_slots_beyond_the_array(cuda_device):
    a, w, bias = workloads.uniform_inputs(8, 512, 512)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    out = torch.empty((8, 512), dtype=torch.float16, device=cuda_device)
    sig = torch.zeros(native.MAX_RANKS, dtype=torch.int64, device=cuda_device)
    status, _ = call_static(da, dw, db, out, sig, native.STATIC_GATHER_SLOTS, 1)
    assert native.STATUS_NAMES[status] == "scratch"
    torch.cuda.synchronize()
    assert int(sig[0]) == 0
