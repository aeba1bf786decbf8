"""GPU parity: the sm_100a kernels against the CPU FP64 oracle.

Every call goes through the C ABI (include/glq.h) via the operator API.  The
gates are the reference's: the seed-7 uniform corpus at
abs <= 0.02 + 0.002 * |ref|; the reference corpus (seed 1729) at
0.003 + 0.005 * |ref| and the fused epilogue at 0.01 + 0.01 * |ref|
(qualification.py:47-56, 95-98).  Output canaries (123-filled guards,
qualification.py:90-94) and NaN-poisoned input storage are checked bit-exact.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import f16
from gemm_lab_qualification_b200 import _native as native
from gemm_lab_qualification_b200 import kernels, workloads
from oracle import reference as oracle

pytestmark = pytest.mark.gpu

U_ATOL, U_RTOL = oracle.UNIFORM_ATOL, oracle.UNIFORM_RTOL


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def guarded_output(m: int, n: int, dtype, device, pitch: int | None = None):
    """Output view inside a 123-filled guard buffer (qualification.py:90-94)."""
    pitch = n if pitch is None else pitch
    rows = max(m, 1)
    guard = torch.full((rows * pitch + 32,), 123, dtype=dtype, device=device)
    out = guard[16:16 + rows * pitch].view(rows, pitch)[:m, :n]
    return guard, out


def assert_guard_intact(guard: torch.Tensor, m: int, n: int, pitch: int | None = None):
    pitch = n if pitch is None else pitch
    g = guard.cpu()
    assert (g[:16] == 123).all() and (g[-16:] == 123).all(), "output canary overwritten"
    if pitch > n and m > 0:
        body = g[16:16 + m * pitch].view(m, pitch)
        assert (body[:, n:] == 123).all(), "row padding of the output overwritten"


@pytest.fixture(autouse=True)
def clean_error_word(cuda_device):
    native.device_error(clear=True)
    yield
    assert native.device_error(clear=True) == 0, "a bounded in-kernel wait expired"


# ------------------------------------------------------------------ headline sweep (M = 1..128, N = K = 4096)

@pytest.mark.parametrize("m", [1, 8, 32, 128])
def test_uniform_sweep_fused(cuda_device, golden, m):
    arrays, _ = golden
    a, w, bias = workloads.uniform_inputs(m, 4096, 4096)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    guard, out = guarded_output(m, 4096, torch.float16, cuda_device)
    kernels.triton_bias_silu_into(da, dw.t(), db, out)
    path = kernels.last_path()
    assert path == (("gemv_m1", 1) if m == 1 else ("tc_splitk", 8 if m <= 32 else 4))
    torch.cuda.synchronize()
    expected = oracle.linear_reference(a, w, bias, silu=True)
    oracle.compare(host(out), expected, U_ATOL, U_RTOL)
    rows = arrays[f"uniform/m{m}/rows"]
    oracle.compare(host(out)[rows], arrays[f"uniform/m{m}/fused_rows"], U_ATOL, U_RTOL)
    assert_guard_intact(guard, m, 4096)


@pytest.mark.parametrize("m", [1, 8, 32, 128])
def test_uniform_sweep_plain(cuda_device, golden, m):
    arrays, _ = golden
    a, w, _ = workloads.uniform_inputs(m, 4096, 4096)
    da, dw = a.to(cuda_device), w.to(cuda_device)
    out = torch.empty((m, 4096), dtype=torch.float16, device=cuda_device)
    kernels.triton_matmul_into(da, dw.t(), out)
    expected = oracle.linear_reference(a, w)
    oracle.compare(host(out), expected, U_ATOL, U_RTOL)
    rows = arrays[f"uniform/m{m}/rows"]
    oracle.compare(host(out)[rows], arrays[f"uniform/m{m}/expected_rows"], U_ATOL, U_RTOL)


def test_uniform_small_golden(cuda_device, golden):
    arrays, _ = golden
    a = torch.from_numpy(f16(arrays["uniform/small/a"]).copy()).to(cuda_device)
    w = torch.from_numpy(f16(arrays["uniform/small/w"]).copy()).to(cuda_device)
    bias = torch.from_numpy(f16(arrays["uniform/small/bias"]).copy()).to(cuda_device)
    out = kernels.triton_bias_silu(a, w.t(), bias)
    assert kernels.last_path()[0] in ("tc_tcgen05", "tc_splitk")
    oracle.compare(host(out), arrays["uniform/small/fused"], U_ATOL, U_RTOL)
    out = kernels.triton_matmul(a, w.t())
    oracle.compare(host(out), arrays["uniform/small/expected"], U_ATOL, U_RTOL)


def test_determinism_bitwise(cuda_device):
    a, w, bias = workloads.uniform_inputs(32, 4096, 4096)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    outs = [kernels.triton_bias_silu(da, dw.t(), db) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))


# ------------------------------------------------------------------ reference corpus

def corpus_cases():
    for shape in workloads.MANIFEST["edges"]:
        for pattern in workloads.MANIFEST["edge_patterns"]:
            for layout in workloads.MANIFEST["layouts"]:
                yield shape, pattern, layout


@pytest.mark.parametrize("shape,pattern,layout", list(corpus_cases()),
                         ids=[f"{s['id']}-{p}-{l}" for s, p, l in corpus_cases()])
def test_reference_corpus(cuda_device, golden, shape, pattern, layout):
    """qualification.check() records (qualification.py:74-99), native kernels."""
    arrays, _ = golden
    key = f"edge/{shape['id']}/{pattern}"
    expected = arrays[key + "/expected"]
    a, b = workloads.inputs(shape, pattern, layout)
    if layout == "strided":
        da = workloads.poisoned_view(a, "strided", cuda_device)
        db = workloads.poisoned_view(b, "strided", cuda_device)
    else:
        da, db = a.to(cuda_device), b.to(cuda_device)
    bases = [t._base if t._base is not None else t for t in (da, db)]
    snapshots = [t.clone() for t in bases]
    m, n = shape["m"], shape["n"]
    guard, out = guarded_output(m, n, torch.float16, cuda_device)
    kernels.triton_matmul_into(da, db, out)
    oracle.compare(host(out), expected)
    assert_guard_intact(guard, m, n)
    path = kernels.last_path()[0]
    if m == 0 or n == 0:
        assert path == "empty"
    elif shape["k"] == 0:
        assert path == "zero_k"
    if m and n:
        bias = workloads.reference_bias(n, device=cuda_device)
        fused = kernels.triton_bias_silu(da, db, bias)
        oracle.compare(host(fused), arrays[key + "/fused"], oracle.FUSED_ATOL, oracle.FUSED_RTOL)
    # inputs and their NaN-poisoned padding are untouched, bit for bit
    for base, snap in zip(bases, snapshots):
        assert torch.equal(base.view(torch.int16), snap.view(torch.int16))


def padded_pitch_view(x: torch.Tensor, device) -> torch.Tensor:
    """Rows padded to a 16-byte pitch (+8 elements), NaN in the gap."""
    rows, cols = x.shape
    pitch = ((cols + 7) // 8) * 8 + 8
    store = torch.full((rows, pitch), float("nan"), dtype=x.dtype, device=device)
    store[:, :cols] = x.to(device)
    return store[:, :cols]


@pytest.mark.parametrize("m,n,k", [(17, 257, 131), (129, 257, 65), (17, 31, 13), (300, 200, 520),
                                   (2, 128, 64), (512, 512, 512)])
def test_tcgen05_tails_in_padded_rows(cuda_device, m, n, k):
    """Ragged M/N/K on the TMA path (OOB zero fill, masked epilogue)."""
    g = torch.Generator().manual_seed(m * 1000 + n + k)
    a = (torch.rand((m, k), generator=g) - .5).half()
    w = (torch.rand((n, k), generator=g) - .5).half()
    bias = (torch.rand((n,), generator=g) - .5).half()
    da = padded_pitch_view(a, cuda_device)
    dw = padded_pitch_view(w, cuda_device)
    db = bias.to(cuda_device)
    pitch = ((n + 7) // 8) * 8 + 8
    guard, out = guarded_output(m, n, torch.float16, cuda_device, pitch=pitch)
    kernels.triton_bias_silu_into(da, dw.t(), db, out)
    path = kernels.last_path()[0]
    assert path in ("tc_tcgen05", "tc_splitk", "tail", "gemv_m1")
    oracle.compare(host(out), oracle.linear_reference(a, w, bias, silu=True), U_ATOL, U_RTOL)
    assert_guard_intact(guard, m, n, pitch=pitch)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("m,n,pitch", [(32, 4096, 4096), (3, 4093, 4093), (70000, 16, 24), (5, 24, 31), (1, 8, 8)])
def test_zero_k_fill(cuda_device, m, n, pitch, dtype):
    """K = 0: every row is epilogue(0 + bias) (16-byte stores down the rows
    when the rows allow, element stores otherwise); nothing outside Y is
    written."""
    g = torch.Generator().manual_seed(m + n)
    bias = ((torch.rand((n,), generator=g) - 0.5) * 8).to(dtype)
    da = torch.empty((m, 0), dtype=dtype, device=cuda_device)
    db = torch.empty((0, n), dtype=dtype, device=cuda_device)
    for fused in (True, False):
        guard, out = guarded_output(m, n, dtype, cuda_device, pitch=pitch)
        if fused:
            kernels.triton_bias_silu_into(da, db, bias.to(cuda_device), out)
        else:
            kernels.triton_matmul_into(da, db, out)
        assert kernels.last_path()[0] == "zero_k"
        torch.cuda.synchronize()
        assert_guard_intact(guard, m, n, pitch=pitch)
        got = out.float().cpu()
        if fused:
            row = torch.nn.functional.silu(bias.float())
            torch.testing.assert_close(got, row.expand(m, n), atol=1e-3, rtol=1e-2)
            assert torch.equal(got, got[:1].expand(m, n)), "rows differ"
        else:
            assert torch.equal(got, torch.zeros((m, n)))


# ------------------------------------------------------------------ boundary probes

def probe_inputs(probe, device):
    m, n, k = probe["m"], probe["n"], probe["k"]
    a, w, bias = workloads.uniform_inputs(m, n, k)
    layout = probe["layout"]
    da, dw = a.to(device), w.to(device)
    if layout == "a_padded":
        da = workloads.poisoned_view(a, "padded", device)
    elif layout == "w_padded":
        dw = workloads.poisoned_view(w, "padded", device)
    elif layout == "a_transposed":
        da = workloads.poisoned_view(a, "transposed", device)
    elif layout == "a_offset":
        da = workloads.poisoned_view(a, "offset", device)
    return a, w, bias, da, dw, bias.to(device)


# K-contiguous rows off 16 bytes (tail K = 4090, a base one element off) run
# the tcgen05 kernel that aligns them itself; a transposed A (no unit stride)
# is copied into the workspace the operator API provides.
EXPECTED_PROBE_PATH = {"zero-m": "empty", "zero-k": "zero_k", "tail-n": "tail", "tail-k": "tc_ldg",
                       "a-row-stride": "tc_splitk", "w-row-stride": "tc_splitk",
                       "a-transposed": "repacked", "misaligned-base": "tc_ldg"}


@pytest.mark.parametrize("probe", workloads.MANIFEST["probes"], ids=[p["id"] for p in workloads.MANIFEST["probes"]])
def test_boundary_probe(cuda_device, probe):
    a, w, bias, da, dw, db = probe_inputs(probe, cuda_device)
    m, n = probe["m"], probe["n"]
    guard, out = guarded_output(m, n, torch.float16, cuda_device)
    before_a = da.clone()
    kernels.triton_bias_silu_into(da, dw.t(), db, out)
    assert kernels.last_path()[0] == EXPECTED_PROBE_PATH[probe["id"]]
    assert_guard_intact(guard, m, n)
    assert torch.equal(da.view(torch.int16), before_a.view(torch.int16)), "input modified"
    if m:
        expected = oracle.linear_reference(a, w, bias, silu=True, samples=8)
        oracle.compare(host(out), expected, U_ATOL, U_RTOL)


# ------------------------------------------------------------------ repacked operands

def aligned_copy(x: torch.Tensor, device) -> torch.Tensor:
    """x ([rows, cols]) in rows padded to a multiple of 8 elements (16 B)."""
    rows, cols = x.shape
    store = torch.full((rows, -(-cols // 8) * 8), float("nan"), dtype=x.dtype, device=device)
    store[:, :cols] = x.to(device)
    return store[:, :cols]


# (id, M, N, K, A layout, B layout); B layouts: "w_nk" = W[N, K].T, "b_kn" =
# B[K, N] row-major, "w_strided" = W[N, K].T with neither stride unit.
REPACK_CASES = [
    ("k131-wide", 64, 2055, 131, "contiguous", "b_kn"),
    ("n4093-b_kn", 32, 4093, 4096, "contiguous", "b_kn"),
    ("m1-n4093-b_kn", 1, 4093, 4096, "contiguous", "b_kn"),
    ("a-transposed", 32, 4096, 4096, "transposed", "w_nk"),
    ("a-transposed-k4090", 32, 4096, 4090, "transposed", "w_nk"),
    ("m509-k4103", 509, 4099, 4103, "contiguous", "w_nk"),
    ("w-strided", 8, 2048, 520, "contiguous", "w_strided"),
    ("m129-odd", 129, 1031, 65, "contiguous", "b_kn"),
]


def layout_operands(case, dtype, device):
    _, m, n, k, a_layout, b_layout = case
    a, w, bias = workloads.uniform_inputs(m, n, k, dtype=dtype)
    da = a.to(device) if a_layout == "contiguous" else workloads.poisoned_view(a, a_layout, device)
    if b_layout == "b_kn":
        b = w.t().contiguous().to(device)
    elif b_layout == "w_strided":
        b = workloads.poisoned_view(w, "strided", device).t()
    else:
        b = w.to(device).t()
    return a, w, bias, da, b


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("case", REPACK_CASES, ids=[c[0] for c in REPACK_CASES])
def test_repacked_matches_aligned_copy(cuda_device, case, dtype):
    """Strided operands, unaligned ones in the lab's B = [K, N], and unaligned
    K-contiguous ones above 128 tokens, with a workspace: the repack kernel's
    aligned copies go through the same tcgen05 / GEMV plan as operands that
    were aligned to begin with, so the bits equal that call's; without a
    workspace the generic kernel runs (or, for K-contiguous rows, the
    tcgen05 kernel that aligns them itself).  Both pass the oracle gate."""
    _, m, n, k, _, b_layout = case
    a, w, bias, da, b = layout_operands(case, dtype, cuda_device)
    b_al = aligned_copy(w.t().contiguous(), cuda_device) if b_layout == "b_kn" else aligned_copy(w, cuda_device).t()
    a_al = aligned_copy(a, cuda_device)
    db = bias.to(cuda_device)
    code = native.dtype_code(dtype)
    need = native.linear_workspace_bytes(code, da.data_ptr(), da.stride(), b.data_ptr(), b.stride(), m, n, k)
    assert need > 0
    assert native.linear_workspace_bytes(code, a_al.data_ptr(), a_al.stride(), b_al.data_ptr(), b_al.stride(),
                                         m, n, k) == 0
    store = torch.full((need + 256,), 255, dtype=torch.uint8, device=cuda_device)
    ws = store[:need]
    epi = native.EPILOGUE_BIAS_SILU
    out_generic = torch.empty((m, n), dtype=dtype, device=cuda_device)
    out_rep, out_al = torch.empty_like(out_generic), torch.empty_like(out_generic)
    path_g, split_g = native.linear(da, b, out_generic, db, epi)
    # no workspace: the generic kernel, or the raw-staged tcgen05 kernel
    assert path_g in ("unaligned", "strided", "tc_ldg")
    path_r, split_r = native.linear(da, b, out_rep, db, epi, workspace=ws)
    assert path_r == "repacked"
    path_a, split_a = native.linear(a_al, b_al, out_al, db, epi)
    assert path_a not in ("unaligned", "strided", "repacked") and split_r == split_a
    torch.cuda.synchronize()
    assert torch.equal(out_rep.view(torch.int16), out_al.view(torch.int16))
    atol, rtol = (U_ATOL, U_RTOL) if dtype == torch.float16 else (0.05, 0.01)
    expected = oracle.linear_reference(a, w, bias, silu=True, samples=8)
    oracle.compare(host(out_rep), expected, atol, rtol)
    oracle.compare(host(out_generic), expected, atol, rtol)
    # A workspace that is too small or misaligned holds no copies: the call
    # takes its no-workspace path.  If that path splits K, the workspace is
    # its FP32 partial buffer, which must be 4-byte aligned.
    assert native.linear(da, b, out_rep, db, epi, workspace=store[:need - 1])[0] == path_g
    if split_g == 1:
        assert native.linear(da, b, out_rep, db, epi, workspace=store[1:need + 1])[0] == path_g
    else:
        with pytest.raises(native.GlqError) as e:
            native.linear(da, b, out_rep, db, epi, workspace=store[1:need + 1])
        assert native.STATUS_NAMES[e.value.status] == "workspace"


# Small problems (<= 2^22 multiply-adds) in layouts the TMA kernels cannot
# address: the small kernel, no workspace, no copy.
SMALL_CASES = [
    ("lab-tail", 17, 257, 131, "contiguous", "b_kn"),
    ("lab-tile-tail", 129, 257, 65, "contiguous", "b_kn"),
    ("lab-odd", 17, 31, 13, "contiguous", "b_kn"),
    ("m1-k131", 1, 257, 131, "contiguous", "w_nk"),
    ("k4090-narrow", 4, 96, 4090, "contiguous", "w_nk"),
    ("a-transposed", 8, 128, 512, "transposed", "w_nk"),
    ("w-strided", 3, 100, 1000, "offset", "w_strided"),
    ("m-rows", 2000, 2, 9, "contiguous", "b_kn"),
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("case", SMALL_CASES, ids=[c[0] for c in SMALL_CASES])
def test_small_kernel(cuda_device, case, dtype):
    _, m, n, k, _, _ = case
    a, w, bias, da, b = layout_operands(case, dtype, cuda_device)
    code = native.dtype_code(dtype)
    assert native.linear_workspace_bytes(code, da.data_ptr(), da.stride(), b.data_ptr(), b.stride(), m, n, k) == 0
    db = bias.to(cuda_device)
    guard, out = guarded_output(m, n, dtype, cuda_device)
    path, split = native.linear(da, b, out, db, native.EPILOGUE_BIAS_SILU)
    assert path in ("unaligned", "strided") and split == 1
    assert_guard_intact(guard, m, n)
    atol, rtol = (U_ATOL, U_RTOL) if dtype == torch.float16 else (0.05, 0.01)
    oracle.compare(host(out), oracle.linear_reference(a, w, bias, silu=True, samples=8), atol, rtol)
    # fixed reduction order: a second call reproduces the bits; no epilogue
    # gives the plain product.
    again = torch.empty_like(out)
    native.linear(da, b, again, db, native.EPILOGUE_BIAS_SILU)
    assert torch.equal(again.view(torch.int16), out.view(torch.int16))
    plain = torch.empty_like(out)
    native.linear(da, b, plain, None, native.EPILOGUE_NONE)
    oracle.compare(host(plain), oracle.linear_reference(a, w, samples=8), atol, rtol)


# K-contiguous rows that TMA cannot address as they are (odd K, a row pitch
# that is not a multiple of 8 elements, a base off 16 bytes), in A, in W or
# in both: the tcgen05 kernel loads them by row class and aligns them in
# shared memory.  (id, M, N, K, A pitch, A offset, W pitch, W offset), pitches
# in elements (None: K rounded up to 8, i.e. an aligned operand), offsets in
# elements from a 256-byte aligned allocation.
RAW_CASES = [
    ("k4090-both", 32, 4096, 4090, 4090, 0, 4090, 0),
    ("k4090-w", 32, 4096, 4090, None, 0, 4090, 0),
    ("a-offset", 32, 4096, 4096, 4096, 1, None, 0),
    ("a-pitch-odd", 8, 4096, 4096, 4097, 0, None, 0),
    ("w-pitch4100", 32, 4096, 4096, None, 0, 4100, 0),
    ("w-offset", 8, 4096, 4096, None, 0, 4096, 1),
    ("both-offset", 16, 2048, 1000, 1000, 3, 1000, 5),
    ("m1-k4090", 1, 4096, 4090, 4090, 0, 4090, 0),
    ("m64-k4095", 64, 2048, 4095, 4095, 0, 4095, 0),
    ("k4095-a8-classes", 32, 4096, 4095, 4095, 0, 4095, 0),
    ("m16-k4095-a8-classes", 16, 2048, 4095, 4095, 0, 4095, 0),
    ("m128-k4090", 128, 4096, 4090, 4090, 0, 4090, 0),
    ("m129-k4090", 129, 1031, 4090, 4090, 0, 4090, 0),
    ("m256-ragged", 256, 777, 1001, 1001, 0, 1001, 0),
    ("m509-odd", 509, 4099, 4103, 4103, 0, 4103, 0),
]


def placed(x: torch.Tensor, pitch, offset: int, device):
    """x ([rows, k]) at `offset` elements into NaN storage, rows `pitch`
    elements apart; returns (storage, view, first element, end element)."""
    rows, k = x.shape
    pitch = -(-k // 8) * 8 if pitch is None else pitch
    store = torch.full((rows * pitch + offset + 64,), float("nan"), dtype=x.dtype, device=device)
    view = store[offset:offset + rows * pitch].view(rows, pitch)[:, :k]
    view.copy_(x.to(device))
    return store, view, offset, offset + (rows - 1) * pitch + k


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("case", RAW_CASES, ids=[c[0] for c in RAW_CASES])
def test_raw_staged_matches_aligned_copy(cuda_device, case, dtype):
    """The tcgen05 kernel on operands it stages raw and aligns itself (path
    tc_ldg, called without a workspace) gives the bits of the same plan on
    16-byte-pitched copies, passes the oracle gate, and reads and writes nothing outside
    the operands (NaN storage around them stays NaN, and no NaN reaches Y)."""
    _, m, n, k, a_pitch, a_off, w_pitch, w_off = case
    a, w, bias = workloads.uniform_inputs(m, n, k, dtype=dtype)
    a_store, da, a_lo, a_hi = placed(a, a_pitch, a_off, cuda_device)
    w_store, dw, w_lo, w_hi = placed(w, w_pitch, w_off, cuda_device)
    db = bias.to(cuda_device)
    code = native.dtype_code(dtype)
    need = native.linear_workspace_bytes(code, da.data_ptr(), da.stride(), dw.data_ptr(), dw.t().stride(), m, n, k)
    # up to 128 tokens no copy is wanted; above, a caller's workspace would
    # hold copies (this call gives none)
    assert (need == 0) == (m <= 128)
    epi = native.EPILOGUE_BIAS_SILU
    out = torch.empty((m, n), dtype=dtype, device=cuda_device)
    out_al = torch.empty_like(out)
    path, split = native.linear(da, dw.t(), out, db, epi)
    assert path == "tc_ldg"
    if m > 1:
        path_al, split_al = native.linear(aligned_copy(a, cuda_device), aligned_copy(w, cuda_device).t(), out_al,
                                          db, epi)
        assert path_al not in ("unaligned", "repacked", "tc_ldg") and split == split_al
    else:
        # M = 1 on aligned rows is a GEMV: check that the call repeats its bits.
        native.linear(da, dw.t(), out_al, db, epi)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), out_al.view(torch.int16))
    assert not torch.isnan(out).any()
    atol, rtol = (U_ATOL, U_RTOL) if dtype == torch.float16 else (0.05, 0.01)
    oracle.compare(host(out), oracle.linear_reference(a, w, bias, silu=True, samples=8), atol, rtol)
    plain = torch.empty_like(out)
    native.linear(da, dw.t(), plain, None, native.EPILOGUE_NONE)
    oracle.compare(host(plain), oracle.linear_reference(a, w, samples=8), atol, rtol)
    for store, lo, hi in ((a_store, a_lo, a_hi), (w_store, w_lo, w_hi)):
        assert torch.isnan(store[:lo]).all() and torch.isnan(store[hi:]).all()


@pytest.mark.parametrize("a_layout,path", [("contiguous", "tc_ldg"), ("transposed", "repacked")])
def test_unaligned_fused_chain_in_a_graph(cuda_device, a_layout, path):
    """Chains of calls on operands TMA cannot address as they are replay
    bit-exactly from a CUDA graph: K = 4090 rows aligned inside the kernel,
    and repacked calls whose workspace comes from torch's caching allocator
    inside the capture."""
    a, w, bias = workloads.uniform_inputs(32, 4090, 4090)
    da = a.to(cuda_device) if a_layout == "contiguous" else workloads.poisoned_view(a, "transposed", cuda_device)
    dw, db = w.to(cuda_device), bias.to(cuda_device)
    y1 = torch.empty((32, 4090), dtype=torch.float16, device=cuda_device)
    y2 = torch.empty_like(y1)

    paths = []

    def chain():
        kernels.triton_bias_silu_into(da, dw.t(), db, y1)
        paths.append(kernels.last_path()[0])
        kernels.triton_bias_silu_into(y1, dw.t(), db, y2)
        paths.append(kernels.last_path()[0])

    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        chain()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    # the second call reads the first one's contiguous K = 4090 output
    assert paths == [path, "tc_ldg"]
    eager = y2.clone()
    oracle.compare(host(y1), oracle.linear_reference(a, w, bias, silu=True, samples=8), U_ATOL, U_RTOL)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    y1.zero_()
    y2.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y2.view(torch.int16), eager.view(torch.int16))


# ------------------------------------------------------------------ split-K probes

@pytest.mark.parametrize("m", [1, 8, 32])
@pytest.mark.parametrize("split", [2, 4, 8])
def test_split_probe(cuda_device, m, split):
    a, w, _ = workloads.uniform_inputs(m, 4096, 4096)
    da, dw = a.to(cuda_device), w.to(cuda_device)
    partial = torch.full((split, m, 4096), float("nan"), dtype=torch.float32, device=cuda_device)
    out = torch.empty((m, 4096), dtype=torch.float16, device=cuda_device)
    kernels.triton_splitk_matmul_into(da, dw.t(), partial, out, split)
    gemv = m == 1 and split == 2
    assert kernels.last_path() == (("gemv_m1" if gemv else "tc_splitk"), split)
    oracle.compare(host(out), oracle.linear_reference(a, w), U_ATOL, U_RTOL)
    granule = 8 if gemv else 64
    parts = oracle.split_partials_reference(a, w.t(), split, granule)
    got = partial.cpu().double().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - parts).max() <= 1e-3 + 1e-4 * np.abs(parts).max()
    # the FP32 merge of the partials in split order reproduces the output bits
    merged = partial[0].clone()
    for s in range(1, split):
        merged = merged + partial[s]
    assert torch.equal(merged.half().view(torch.int16), out.view(torch.int16))


def test_splitk_plan_and_default(cuda_device):
    a, w, _ = workloads.uniform_inputs(8, 4096, 4096)
    da, dw = a.to(cuda_device), w.to(cuda_device)
    plan = kernels.TritonSplitKPlan(da, dw.t(), 8)
    assert plan.workspace_bytes() == 8 * 8 * 4096 * 4
    out = plan()
    oracle.compare(host(out), oracle.linear_reference(a, w), U_ATOL, U_RTOL)
    out2 = kernels.triton_splitk_matmul(da, dw.t())
    assert kernels.last_path() == ("tc_splitk", 4)
    oracle.compare(host(out2), oracle.linear_reference(a, w), U_ATOL, U_RTOL)


# ------------------------------------------------------------------ layouts, dtypes, ops

@pytest.mark.parametrize("m", [1, 8, 32, 128])
def test_reference_layout_b_kn(cuda_device, m):
    """The lab's own B = [K, N] row-major operand (qualification.py:63-64,
    kernels.py:148-171): MN-major W tiles on the tcgen05 path, same gate."""
    a, w, bias = workloads.uniform_inputs(m, 4096, 4096)
    da, dw, dbias = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    db_kn = dw.t().contiguous()
    fused = kernels.triton_bias_silu(da, db_kn, dbias)
    assert kernels.last_path()[0] == "tc_kn"
    oracle.compare(host(fused), oracle.linear_reference(a, w, bias, silu=True), U_ATOL, U_RTOL)
    guard, out = guarded_output(m, 4096, torch.float16, cuda_device)
    kernels.triton_matmul_into(da, db_kn, out)
    assert kernels.last_path()[0] == "tc_kn"
    oracle.compare(host(out), oracle.linear_reference(a, w), U_ATOL, U_RTOL)
    assert_guard_intact(guard, m, 4096)
    if m > 1:
        # Same tiles, split and MMA sequence as the K-contiguous operand.
        fused_k = kernels.triton_bias_silu(da, dw.t(), dbias)
        assert kernels.last_path()[1] == kernels.planned_path(da, db_kn)[1]
        assert torch.equal(fused.view(torch.int16), fused_k.view(torch.int16))


@pytest.mark.parametrize("m,n,k", [(17, 257, 131), (129, 257, 65), (17, 31, 13), (300, 200, 520),
                                   (2, 128, 64), (1, 4093, 4096), (512, 512, 512)])
def test_b_kn_tails_in_padded_rows(cuda_device, m, n, k):
    """B = [K, N] with ragged M/N/K in 16-byte-pitched rows (OOB zero fill)."""
    g = torch.Generator().manual_seed(m * 7919 + n * 31 + k)
    a = (torch.rand((m, k), generator=g) - .5).half()
    w = (torch.rand((n, k), generator=g) - .5).half()
    bias = (torch.rand((n,), generator=g) - .5).half()
    da = padded_pitch_view(a, cuda_device)
    db_kn = padded_pitch_view(w.t().contiguous(), cuda_device)
    pitch = ((n + 7) // 8) * 8 + 8
    guard, out = guarded_output(m, n, torch.float16, cuda_device, pitch=pitch)
    kernels.triton_bias_silu_into(da, db_kn, bias.to(cuda_device), out)
    ragged = n % 128 != 0 or k % 64 != 0
    assert kernels.last_path()[0] == ("tail" if ragged else "tc_kn")
    oracle.compare(host(out), oracle.linear_reference(a, w, bias, silu=True), U_ATOL, U_RTOL)
    assert_guard_intact(guard, m, n, pitch=pitch)


@pytest.mark.parametrize("m", [1, 8, 32])
@pytest.mark.parametrize("split", [2, 4, 8])
def test_b_kn_split_probe(cuda_device, m, split):
    """Split-K on B = [K, N]: partial write-back and the fixed-order merge."""
    a, w, _ = workloads.uniform_inputs(m, 4096, 4096)
    da, db_kn = a.to(cuda_device), w.t().contiguous().to(cuda_device)
    partial = torch.full((split, m, 4096), float("nan"), dtype=torch.float32, device=cuda_device)
    out = torch.empty((m, 4096), dtype=torch.float16, device=cuda_device)
    kernels.triton_splitk_matmul_into(da, db_kn, partial, out, split)
    assert kernels.last_path() == ("tc_kn", split)
    oracle.compare(host(out), oracle.linear_reference(a, w), U_ATOL, U_RTOL)
    merged = partial[0].clone()
    for s in range(1, split):
        merged = merged + partial[s]
    assert torch.equal(merged.half().view(torch.int16), out.view(torch.int16))


def test_native_launch_surface_b_kn(cuda_device):
    """glq_matmul / glq_splitk_matmul: the lab's launch_X(a, b, c, m, n, k, stream)
    with B = [K, N] row-major (csrc/ptx_mma.cuh:220-965)."""
    lib = native.library()
    m, n, k = 32, 4096, 4096
    a, w, _ = workloads.uniform_inputs(m, n, k)
    da, db_kn = a.to(cuda_device), w.t().contiguous().to(cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    c = torch.empty((m, n), dtype=torch.float16, device=cuda_device)
    assert lib.glq_matmul(0, da.data_ptr(), db_kn.data_ptr(), c.data_ptr(), m, n, k, stream) == 0
    c2 = torch.empty_like(c)
    partial = torch.empty((4, m, n), dtype=torch.float32, device=cuda_device)
    assert lib.glq_splitk_matmul(0, da.data_ptr(), db_kn.data_ptr(), c2.data_ptr(), m, n, k,
                                 partial.data_ptr(), 4, stream) == 0
    torch.cuda.synchronize()
    expected = oracle.linear_reference(a, w)
    oracle.compare(host(c), expected, U_ATOL, U_RTOL)
    oracle.compare(host(c2), expected, U_ATOL, U_RTOL)


@pytest.mark.parametrize("m", [1, 32])
def test_bf16(cuda_device, m):
    a, w, bias = workloads.uniform_inputs(m, 4096, 4096, dtype=torch.bfloat16)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    out = kernels.triton_bias_silu(da, dw.t(), db)
    expected = oracle.linear_reference(a, w, bias, silu=True)
    oracle.compare(host(out), expected, 0.05, 0.01)


def test_custom_ops_and_plans(cuda_device):
    a, w, bias = workloads.uniform_inputs(32, 4096, 4096)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    ref_plain = oracle.linear_reference(a, w)
    ref_fused = oracle.linear_reference(a, w, bias, silu=True)
    oracle.compare(host(torch.ops.gemm_lab.triton_matmul(da, dw.t())), ref_plain, U_ATOL, U_RTOL)
    oracle.compare(host(torch.ops.gemm_lab.triton_splitk_matmul(da, dw.t())), ref_plain, U_ATOL, U_RTOL)
    oracle.compare(host(torch.ops.gemm_lab.adaptive_matmul(da, dw.t())), ref_plain, U_ATOL, U_RTOL)
    oracle.compare(host(torch.ops.gemm_lab.triton_bias_silu(da, dw.t(), db)), ref_fused, U_ATOL, U_RTOL)
    oracle.compare(host(torch.ops.gemm_lab.adaptive_bias_silu(da, dw.t(), db)), ref_fused, U_ATOL, U_RTOL)
    oracle.compare(host(kernels.TritonMatmulPlan(da, dw.t())()), ref_plain, U_ATOL, U_RTOL)
    oracle.compare(host(kernels.TritonBiasSiluPlan(da, dw.t(), db)()), ref_fused, U_ATOL, U_RTOL)
    oracle.compare(host(kernels.AdaptiveMatmulPlan(da, dw.t())()), ref_plain, U_ATOL, U_RTOL)


def test_bias_only_epilogue_and_streams(cuda_device):
    a, w, bias = workloads.uniform_inputs(16, 1024, 2048)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        out = torch.empty((16, 1024), dtype=torch.float16, device=cuda_device)
        kernels.linear_into(da, dw.t(), out, db)
    stream.synchronize()
    expected = oracle.linear_reference(a, w) + bias.double().numpy()[None, :]
    oracle.compare(host(out), expected, U_ATOL, U_RTOL)


@pytest.mark.parametrize("m", [1, 32])
def test_launch_modes_bitwise_identical(cuda_device, m):
    """PDL on/off and the static-weights flag change scheduling, never results."""
    a, w, bias = workloads.uniform_inputs(m, 4096, 4096)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    outs = []
    for opts in (dict(pdl=False), dict(), dict(static_weights=True)):
        with kernels.launch_options(**opts):
            # back-to-back calls so dependent launches really overlap
            for _ in range(4):
                out = kernels.triton_bias_silu(da, dw.t(), db)
        outs.append(out)
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    oracle.compare(host(outs[0]), oracle.linear_reference(a, w, bias, silu=True), U_ATOL, U_RTOL)


def test_pdl_chain_respects_dependencies(cuda_device):
    """y1 = f(A, W1) feeds the next call as its A; with PDL the second call
    must still see the finished y1 (griddepcontrol.wait before reading A)."""
    a, w1, b1 = workloads.uniform_inputs(32, 4096, 4096)
    _, w2, b2 = workloads.uniform_inputs(32, 4096, 4096, seed=8)
    da, dw1, db1, dw2, db2 = (t.to(cuda_device) for t in (a, w1, b1, w2, b2))
    with kernels.launch_options(static_weights=True):
        y1 = kernels.triton_bias_silu(da, dw1.t(), db1)
        y2 = kernels.triton_bias_silu(y1, dw2.t(), db2)
    torch.cuda.synchronize()
    ref1 = kernels.triton_bias_silu(da, dw1.t(), db1)
    with kernels.launch_options(pdl=False):
        ref2 = kernels.triton_bias_silu(ref1, dw2.t(), db2)
    torch.cuda.synchronize()
    assert torch.equal(y1.view(torch.int16), ref1.view(torch.int16))
    assert torch.equal(y2.view(torch.int16), ref2.view(torch.int16))
    expected = oracle.linear_reference(host(y1).astype(np.float16), w2, b2, silu=True)
    oracle.compare(host(y2), expected, U_ATOL, U_RTOL)


@pytest.mark.parametrize("m,n", [(4096, 3072), (4000, 3000)])
def test_prefill_256x256_tiles(cuda_device, m, n):
    """Prefill-sized M on enough output tiles for 256 x 256 tiles (two M = 128
    MMAs per K step), token tiles fastest in launch order; ragged M and N."""
    g = torch.Generator().manual_seed(m + n)
    a = (torch.rand((m, 1024), generator=g) - .5).half()
    w = (torch.rand((n, 1024), generator=g) - .5).half()
    bias = (torch.rand((n,), generator=g) - .5).half()
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    out = kernels.triton_bias_silu(da, dw.t(), db)
    assert kernels.last_path() == ("tc_tcgen05" if n % 128 == 0 else "tail", 1)
    oracle.compare(host(out), oracle.linear_reference(a, w, bias, silu=True, samples=8), U_ATOL, U_RTOL)
    out_kn = kernels.triton_matmul(da, dw.t().contiguous())
    oracle.compare(host(out_kn), oracle.linear_reference(a, w, samples=8), U_ATOL, U_RTOL)


@pytest.mark.parametrize("m", [1, 32, 128])
def test_cuda_graph_capture_and_replay(cuda_device, m):
    """A dependent chain of three layers (GEMV / split-K cluster / tile paths,
    programmatic dependent launch between them) captured once into a CUDA
    graph and replayed twice reproduces the eager bits."""
    a, w1, b1 = workloads.uniform_inputs(m, 4096, 4096)
    _, w2, b2 = workloads.uniform_inputs(m, 4096, 4096, seed=8)
    _, w3, b3 = workloads.uniform_inputs(m, 4096, 4096, seed=9)
    da, dw1, db1, dw2, db2, dw3, db3 = (t.to(cuda_device) for t in (a, w1, b1, w2, b2, w3, b3))
    y1 = torch.empty((m, 4096), dtype=torch.float16, device=cuda_device)
    y2, y3 = torch.empty_like(y1), torch.empty_like(y1)

    def chain():
        kernels.triton_bias_silu_into(da, dw1.t(), db1, y1)
        kernels.triton_bias_silu_into(y1, dw2.t(), db2, y2)
        kernels.triton_bias_silu_into(y2, dw3.t(), db3, y3)

    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        chain()  # warm-up: per-device set-up happens outside the capture
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    eager = y3.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    for _ in range(2):
        y1.zero_()
        y2.zero_()
        y3.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y3.view(torch.int16), eager.view(torch.int16))


@pytest.mark.parametrize("m", [8, 32])
def test_wide_layer_256_row_tiles(cuda_device, m):
    """M <= 32 on N >= 8192 takes 256-row W tiles (two accumulators)."""
    a, w, bias = workloads.uniform_inputs(m, 8192, 2048)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    out = kernels.triton_bias_silu(da, dw.t(), db)
    assert kernels.last_path() == ("tc_splitk", 4)
    oracle.compare(host(out), oracle.linear_reference(a, w, bias, silu=True), U_ATOL, U_RTOL)
    # ragged N on the same tiles
    out = kernels.triton_bias_silu(da, dw[:8000].t(), db[:8000])
    assert kernels.last_path()[0] == "tail"
    oracle.compare(host(out), oracle.linear_reference(a, w[:8000], bias[:8000], silu=True), U_ATOL, U_RTOL)


@pytest.mark.parametrize("m", [1, 32, 128, 512])
@pytest.mark.parametrize("n,k", [(11008, 4096), (4096, 11008)])
def test_mlp_shapes(cuda_device, m, n, k):
    """The MLP shapes the lab's adaptive_bias_silu_path gates on (kernels.py:295,
    4096 <-> 11008), both weight layouts, against the FP64 oracle."""
    a, w, bias = workloads.uniform_inputs(m, n, k)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    expected = oracle.linear_reference(a, w, bias, silu=True, samples=8)
    out = kernels.adaptive_bias_silu(da, dw.t(), db)
    oracle.compare(host(out), expected, U_ATOL, U_RTOL)
    out_kn = kernels.triton_bias_silu(da, dw.t().contiguous(), db)
    assert kernels.last_path()[0] == "tc_kn"
    oracle.compare(host(out_kn), expected, U_ATOL, U_RTOL)


def test_column_parallel_single_rank(cuda_device, tmp_path):
    """The sharded layer on a one-rank NCCL group equals the unsharded call."""
    import torch.distributed as dist
    from gemm_lab_qualification_b200 import sharded
    store = dist.FileStore(str(tmp_path / "store"), 1)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, device_id=cuda_device)
    try:
        a, w, bias = workloads.uniform_inputs(32, 4096, 4096)
        layer = sharded.ColumnParallelLinear(w, bias, "silu", device=cuda_device)
        y = layer(a.to(cuda_device))
        torch.cuda.synchronize()
        oracle.compare(host(y), oracle.linear_reference(a, w, bias, silu=True), U_ATOL, U_RTOL)
    finally:
        dist.destroy_process_group()
