"""The C ABI of libglq.so without a GPU: symbols, names, planning, validation.

Every symbol include/glq.h declares must be exported; path planning
(glq_plan) and workspace sizing are pure host functions and are checked here
against the rules the kernels rely on.  No compute call runs on the CPU:
a real launch request returns GLQ_ERR_DEVICE when there is no sm_100a GPU.
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from gemm_lab_qualification_b200 import _native as native

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "glq.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(glq_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = native.library()
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(native.SIGNATURES), "binding and header disagree"
    out = subprocess.run(["nm", "-D", "--defined-only", str(native.LIBRARY_PATH)], capture_output=True, text=True)
    if out.returncode == 0:
        exported = set(re.findall(r"\b(glq_[a-z0-9_]+)\b", out.stdout))
        assert set(names) <= exported


def test_abi_version_and_target():
    lib = native.library()
    assert lib.glq_abi_version() == 3
    assert lib.glq_build_target() == b"sm_100a"


def test_path_and_status_names():
    assert [native.path_name(i) for i in range(len(native.PATHS))] == list(native.PATHS)
    assert native.path_name(99) == "unknown"
    for status in range(len(native.STATUS_NAMES)):
        assert native.status_string(status)
    assert native.status_string(0) == "ok"


def plan(m, n, k, a_strides=None, b_strides=None, a_ptr=0, b_ptr=0, split=0, ldy=None, dtype=0, sms=148):
    a_strides = a_strides or (k, 1)
    b_strides = b_strides or (1, k)  # W[N, K].T: the K-contiguous fast layout
    return native.plan(dtype, a_ptr, a_strides, b_ptr, b_strides, ldy if ldy is not None else n, m, n, k,
                       split, sms)


@pytest.mark.parametrize("m,expected", [(1, ("gemv_m1", 1)), (8, ("tc_splitk", 8)), (32, ("tc_splitk", 8)),
                                        (128, ("tc_splitk", 4))])
def test_plan_decode_sweep(m, expected):
    assert plan(m, 4096, 4096) == expected


def test_plan_boundaries():
    assert plan(0, 4096, 4096)[0] == "empty"
    assert plan(32, 0, 4096)[0] == "empty"
    assert plan(32, 4096, 0)[0] == "zero_k"
    assert plan(32, 4093, 4096)[0] == "tail"
    # K = 4090 contiguous: row pitch 8180 B is not a multiple of 16, so
    # neither operand is a TMA source as it is; the tcgen05 kernel loads both
    # by row class and aligns them in shared memory.
    assert plan(32, 4096, 4090) == ("tc_ldg", 8)
    # K = 4090 in rows padded to 4096 elements: TMA with OOB zero fill.
    assert plan(32, 4096, 4090, a_strides=(4096, 1), b_strides=(1, 4096))[0] == "tail"
    # padded rows (K + 8) keep 16-byte pitches.
    assert plan(32, 4096, 4096, a_strides=(4104, 1))[0] == "tc_splitk"
    assert plan(32, 4096, 4096, b_strides=(1, 4104))[0] == "tc_splitk"
    # transposed A -> generic kernel.
    assert plan(32, 4096, 4096, a_strides=(1, 32))[0] == "strided"
    # the reference's own B = [K, N] row-major layout -> MN-major tensor-core path.
    assert plan(32, 4096, 4096, b_strides=(4096, 1)) == ("tc_kn", 8)
    assert plan(1, 4096, 4096, b_strides=(4096, 1)) == ("tc_kn", 8)
    assert plan(128, 4096, 4096, b_strides=(4096, 1)) == ("tc_kn", 4)
    # B = [K, N] with a ragged N in 16-byte-pitched rows: tails on the same kernel.
    assert plan(17, 257, 131, a_strides=(136, 1), b_strides=(264, 1)) == ("tail", 1)
    assert plan(32, 4093, 4096, b_strides=(4096, 1)) == ("tail", 8)
    # B = [K, N] rows not 16-byte pitched (N = 4093 contiguous) -> generic kernel.
    assert plan(32, 4093, 4096, b_strides=(4093, 1))[0] == "unaligned"
    # neither operand dimension contiguous -> generic kernel.
    assert plan(32, 4096, 4096, b_strides=(2, 8192))[0] == "strided"
    # K-contiguous rows that TMA cannot address (odd base, pitch or K) in A,
    # W or both: the tcgen05 kernel stages them raw and aligns them.
    assert plan(32, 4096, 4096, a_ptr=2) == ("tc_ldg", 8)
    assert plan(1, 4096, 4096, b_ptr=2)[0] == "tc_ldg"
    assert plan(32, 4096, 4090, a_strides=(4096, 1)) == ("tc_ldg", 8)
    assert plan(32, 4096, 4096, b_strides=(1, 4100)) == ("tc_ldg", 8)
    assert plan(128, 4096, 4096, b_strides=(1, 4097)) == ("tc_ldg", 4)
    assert plan(509, 4099, 4103)[0] == "tc_ldg"
    # rows so short that 8 row classes cannot keep them apart (C * pitch must
    # reach K + 8) leave the tensor-core path.
    assert plan(4096, 4096, 1, a_strides=(1, 1), b_strides=(1, 1))[0] == "unaligned"
    assert plan(4096, 4096, 3, a_strides=(3, 1), b_strides=(1, 3))[0] == "tc_ldg"


@pytest.mark.parametrize("m", [1, 8, 32])
@pytest.mark.parametrize("split", [2, 4, 8])
def test_plan_forced_split(m, split):
    path, s = plan(m, 4096, 4096, split=split)
    assert s == split
    # M = 1: the GEMV splits in two; larger forced splits use the tcgen05 kernel.
    assert path == ("gemv_m1" if m == 1 and split == 2 else "tc_splitk")


def test_plan_split_clamped_to_k_blocks():
    # K = 100 has two 64-wide blocks: a forced split of 8 becomes 2.
    assert plan(32, 4096, 100, a_strides=(104, 1), b_strides=(1, 104), split=8) == ("tail", 2)
    # one block: no split possible.
    assert plan(32, 4096, 64, split=8) == ("tc_tcgen05", 1)


def test_plan_auto_split_tracks_sm_count():
    # 32 tiles: two CTAs per SM with an 8-way split (256 CTAs) when 148 SMs.
    assert plan(32, 4096, 4096, sms=148) == ("tc_splitk", 8)
    assert plan(32, 4096, 4096, sms=64) == ("tc_splitk", 2)
    assert plan(32, 4096, 4096, sms=32) == ("tc_tcgen05", 1)
    assert plan(128, 4096, 4096, sms=148) == ("tc_splitk", 4)
    # M <= 32 on N >= 8192: 256-row W tiles, 32 tiles -> split 4.
    assert plan(32, 8192, 8192) == ("tc_splitk", 4)
    # prefill: 16 x 8 = 128 tiles already fill the device.
    assert plan(4096, 1024, 8192) == ("tc_tcgen05", 1)
    # sharded MLP slice 28672 / 8 = 3584 rows: 28 tiles -> two per SM, split 8.
    assert plan(32, 3584, 8192) == ("tc_splitk", 8)
    assert plan(128, 3584, 8192) == ("tc_splitk", 4)


def test_plan_rejects_bad_arguments():
    with pytest.raises(native.GlqError) as e:
        plan(32, 4096, 4096, split=9)
    assert e.value.status == 3
    with pytest.raises(native.GlqError) as e:
        plan(-1, 4096, 4096)
    assert e.value.status == 2
    with pytest.raises(native.GlqError) as e:
        plan(32, 4096, 4096, dtype=7)
    assert e.value.status == 1
    with pytest.raises(native.GlqError) as e:
        plan(32, 4096, 4096, ldy=100)
    assert e.value.status == 5


def test_workspace_bytes():
    assert native.workspace_bytes(32, 4096, 4096, 0) == 8 * 32 * 4096 * 4
    assert native.workspace_bytes(128, 4096, 4096, 0) == 4 * 128 * 4096 * 4
    assert native.workspace_bytes(8, 4096, 4096, 8) == 8 * 8 * 4096 * 4
    # M = 1: the K-contiguous GEMV does not split, B = [K, N] takes the
    # tensor-core path with an 8-way split; the size covers both layouts.
    assert native.workspace_bytes(1, 4096, 4096, 0) == 8 * 1 * 4096 * 4
    assert native.workspace_bytes(1, 4096, 4096, 4) == 4 * 4096 * 4
    assert native.workspace_bytes(32, 4096, 4096, 1) == 0
    assert native.workspace_bytes(0, 4096, 4096, 4) == 0
    assert native.workspace_bytes(32, 4096, 4096, 9) == 0


def repack_bytes(m, n, k, a_strides=None, b_strides=None, a_ptr=0, b_ptr=0):
    a_strides = a_strides or (k, 1)
    b_strides = b_strides or (1, k)
    return native.linear_workspace_bytes(native.DTYPE_F16, a_ptr, a_strides, b_ptr, b_strides, m, n, k)


def padded(rows, cols):
    """Bytes of one aligned copy: rows of ceil(cols / 8) * 8 FP16, 256-B rounded."""
    return -(-rows * (-(-cols // 8) * 8) * 2 // 256) * 256


def test_linear_workspace_bytes():
    # TMA-addressable operands need no copy.
    assert repack_bytes(32, 4096, 4096) == 0
    assert repack_bytes(32, 4096, 4096, b_strides=(4096, 1)) == 0
    assert repack_bytes(32, 4096, 4090, a_strides=(4096, 1), b_strides=(1, 4096)) == 0
    # K-contiguous rows off 16 bytes (K = 4090 contiguous, a base two bytes
    # off) in A or in W = B^T: the tcgen05 kernel aligns them itself, no copy.
    assert repack_bytes(32, 4096, 4090) == 0
    assert repack_bytes(32, 4096, 4096, a_ptr=2) == 0
    assert repack_bytes(1, 4096, 4096, b_ptr=2) == 0
    # above 128 tokens they are copied when the workspace allows (every token
    # tile would re-align the same W tiles).
    assert repack_bytes(509, 4099, 4103) == padded(509, 4103) + padded(4099, 4103)
    assert repack_bytes(129, 4096, 4096, a_ptr=2) == padded(129, 4096)
    assert repack_bytes(128, 4096, 4096, a_ptr=2) == 0
    # a transposed A (no unit stride) is copied, and only A.
    assert repack_bytes(32, 4096, 4096, a_strides=(1, 32)) == padded(32, 4096)
    # with a transposed A, a misaligned W is copied too (the copies then run
    # the TMA kernels).
    assert repack_bytes(32, 4096, 4090, a_strides=(1, 32)) == padded(32, 4090) + padded(4096, 4090)
    # B = [K, N] with N = 4093: the copy keeps B N-contiguous ([K, N] rows).
    assert repack_bytes(32, 4093, 4096, b_strides=(4093, 1)) == padded(4096, 4093)
    # no unit stride in B: copied K-contiguous.
    assert repack_bytes(32, 4096, 4096, b_strides=(2, 8192)) == padded(4096, 4096)
    # a wider tail shape, both operands row-major with odd pitches.
    assert repack_bytes(64, 2055, 131, b_strides=(2055, 1)) == padded(64, 131) + padded(131, 2055)
    # small problems (<= 2^22 multiply-adds, e.g. the lab's 17 x 257 x 131
    # tail) run the small kernel on the operands as they are: no copy.
    assert repack_bytes(17, 257, 131, b_strides=(257, 1)) == 0
    assert repack_bytes(1, 4096, 1023) == 0
    assert repack_bytes(1, 4096, 1025) == 0
    assert repack_bytes(1, 4093, 4096, b_strides=(4093, 1)) == padded(4096, 4093)
    # nothing to compute, or invalid arguments.
    assert repack_bytes(0, 4096, 4090) == 0
    assert repack_bytes(32, 4096, 0) == 0
    assert native.linear_workspace_bytes(7, 0, (4090, 1), 0, (1, 4090), 32, 4096, 4090) == 0


def repack_chunk(row: bytes, col0: int, cols: int, base: int) -> bytes:
    """Host restatement of one 16-byte output chunk of repack_rows_kernel.

    `row` holds the bytes of the aligned granules around a row that starts at
    address `base` (the row's first byte is row[base % 16]); the chunk of
    columns col0 .. col0 + 7 comes from the granule holding its first byte
    and the next one, shifted by the byte offset, columns >= cols zeroed.
    """
    first = base + 2 * col0
    g0 = first - first % 16
    shift = first - g0
    end = base + 2 * cols
    origin = base - base % 16  # address of row[0]
    lo = row[g0 - origin:g0 - origin + 16]
    hi = row[g0 + 16 - origin:g0 + 32 - origin] if shift and g0 + 16 < end else bytes(16)
    words = [int.from_bytes((lo + hi)[4 * i:4 * i + 4], "little") for i in range(8)]
    q, bits = shift >> 2, (shift & 3) * 8
    pick = [words[j + q] for j in range(5)]
    out = [((pick[j + 1] << 32 | pick[j]) >> bits) & 0xFFFFFFFF for j in range(4)]
    valid = cols - col0
    for j in range(4):
        if 2 * j >= valid:
            out[j] = 0
        elif 2 * j + 1 >= valid:
            out[j] &= 0xFFFF
    return b"".join(w.to_bytes(4, "little") for w in out)


@pytest.mark.parametrize("cols", [1, 7, 8, 9, 131, 4090])
def test_repack_window_restatement(cols):
    """Every byte offset of a row start (even offsets for 2-byte elements and
    odd ones too) gives the row's elements, zero-padded to a multiple of 8."""
    rng = np.random.default_rng(cols)
    for base in range(1024, 1040):
        start = base % 16
        span = -(-(start + 2 * cols) // 16) * 16 + 16
        row = rng.integers(0, 256, size=span, dtype=np.uint8).tobytes()
        expected = row[start:start + 2 * cols] + bytes(2 * (-(-cols // 8) * 8 - cols))
        got = b"".join(repack_chunk(row, c, cols, base) for c in range(0, cols, 8))
        assert got == expected


def test_linear_validation_precedes_device_use():
    lib = native.library()
    path = ctypes.c_int(-1)
    split = ctypes.c_int(-1)
    # bad dtype / epilogue / split / shapes / null pointers: no device needed.
    assert lib.glq_linear(5, None, 0, 1, None, 1, 0, None, 0, None, 0, 1, 1, 1, 0, None, 0, None, None, None) == 1
    assert lib.glq_linear(0, None, 0, 1, None, 1, 0, None, 9, None, 0, 1, 1, 1, 0, None, 0, None, None, None) == 1
    assert lib.glq_linear(0, None, 0, 1, None, 1, 0, None, 0, None, 0, 1, 1, 1, 9, None, 0, None, None, None) == 3
    assert lib.glq_linear(0, None, 0, 1, None, 1, 0, None, 0, None, 0, -1, 1, 1, 0, None, 0, None, None, None) == 2
    assert lib.glq_linear(0, None, 0, 1, None, 1, 0, None, 0, None, 0, 1, 1, 1, 0, None, 0, None, None, None) == 1
    # unknown flag bits
    assert lib.glq_linear_ex(0, None, 0, 1, None, 1, 0, None, 0, None, 0, 1, 1, 1, 0, None, 0, None, 1 << 7,
                             None, None) == 1
    # bias+SiLU without a bias pointer
    assert lib.glq_linear(0, 16, 1, 1, 16, 1, 1, None, 2, 16, 1, 1, 1, 1, 0, None, 0, None, None, None) == 1
    # 16-bit element pointers at odd addresses (A, B, bias, Y in turn)
    for a_ptr, b_ptr, bias_ptr, y_ptr in ((17, 16, 16, 16), (16, 17, 16, 16), (16, 16, 17, 16), (16, 16, 16, 17)):
        assert lib.glq_linear(0, a_ptr, 8, 1, b_ptr, 1, 8, bias_ptr, 2, y_ptr, 8, 2, 8, 8, 0, None, 0, None,
                              None, None) == 1
    # empty problems succeed without touching a device and report "empty"
    assert lib.glq_linear(0, None, 0, 1, None, 1, 0, None, 0, None, 0, 0, 8, 8, 0, None, 0, None,
                          ctypes.byref(path), ctypes.byref(split)) == 0
    assert native.PATHS[path.value] == "empty" and split.value == 1


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device status on a GPU-less host")
def test_compute_call_without_gpu_fails_loudly():
    lib = native.library()
    status = lib.glq_linear(0, 16, 8, 1, 16, 1, 8, None, 0, 32, 8, 2, 8, 8, 0, None, 0, None, None, None)
    assert status == 7  # GLQ_ERR_DEVICE: no CPU fallback exists
    a = torch.zeros(2, 8, dtype=torch.float16)
    with pytest.raises(native.GlqError):
        native.linear(a, a.t(), torch.empty(2, 2, dtype=torch.float16))


def test_operator_api_contract_errors_on_cpu():
    """ValueError contract of kernels.py:132-145 / 396-409."""
    from gemm_lab_qualification_b200 import kernels
    a = torch.zeros(4, 8, dtype=torch.float16)
    b = torch.zeros(8, 3, dtype=torch.float16)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        kernels.triton_matmul(a, b)
    with pytest.raises(ValueError, match="rank-2"):
        kernels.triton_matmul(a[0], b)
    with pytest.raises(ValueError, match="incompatible dimensions"):
        kernels.triton_matmul(a, b[:4])
    with pytest.raises(ValueError, match="split_k must be 2, 4, or 8"):
        kernels.triton_splitk_matmul_into(a, b, None, None, split_k=3)
    with pytest.raises(ValueError, match="split_k must be 2, 4, or 8"):
        kernels.TritonSplitKPlan(a, b, 16)


def test_custom_ops_registered_with_fake_kernels():
    from gemm_lab_qualification_b200 import kernels  # noqa: F401  (registers the ops)
    for name in ["triton_matmul", "triton_splitk_matmul", "triton_adaptive_matmul", "adaptive_matmul",
                 "triton_bias_silu", "adaptive_bias_silu"]:
        assert hasattr(torch.ops.gemm_lab, name), name
    with torch._subclasses.fake_tensor.FakeTensorMode():
        a = torch.empty(4, 8, dtype=torch.float16, device="cuda")
        b = torch.empty(8, 3, dtype=torch.float16, device="cuda")
        bias = torch.empty(3, dtype=torch.float16, device="cuda")
        assert torch.ops.gemm_lab.triton_matmul(a, b).shape == (4, 3)
        assert torch.ops.gemm_lab.triton_bias_silu(a, b, bias).shape == (4, 3)


def test_adaptive_path_names_native_kernel():
    from gemm_lab_qualification_b200 import kernels
    assert kernels.adaptive_path(8, 4096, 4096, torch.float16) == "tc_splitk"
    assert kernels.adaptive_path(1, 4096, 4096) == "gemv_m1"
    # MLP up-projection: 43 tiles of 256 rows, split 3 -> 129 CTAs.
    assert kernels.adaptive_bias_silu_path(8, 11008, 4096, torch.float16) == "tc_splitk"
    assert kernels.adaptive_path(8, 11008, 4096, torch.float16) == "tc_splitk"


def gather_status(**over):
    """glq_linear_gather with plausible host-side arguments; pointers are fake
    (non-null) because every check below fails before any device access."""
    lib = native.library()
    VP = ctypes.c_void_p
    args = dict(dtype=0, a=16, lda=4096, acs=1, b=16, bks=1, bns=4096, bias=16, epi=2, ldy=8192, off=4096,
                m=32, n=4096, k=4096, split=0, rank=1, world=2, counter=16, epoch=1, flags=0)
    args.update(over)
    ys = (VP * 2)(16, 17 if over.get("ys_odd") else 16) if over.get("ys", True) else None
    sigs = (VP * 2)(16, 16) if over.get("sigs", True) else None
    counter = ctypes.cast(VP(args["counter"]), ctypes.POINTER(ctypes.c_uint)) if args["counter"] else None
    return lib.glq_linear_gather(args["dtype"], args["a"], args["lda"], args["acs"], args["b"], args["bks"],
                                 args["bns"], args["bias"], args["epi"], ys, args["ldy"], args["off"], args["m"],
                                 args["n"], args["k"], args["split"], args["rank"], args["world"], sigs, counter,
                                 args["epoch"], None, args["flags"], None, None)


def test_gather_argument_validation():
    assert gather_status(world=0) == 1
    assert gather_status(world=9) == 1
    assert gather_status(rank=2) == 1
    assert gather_status(rank=-1) == 1
    assert gather_status(epoch=0) == 1
    assert gather_status(counter=0) == 1
    assert gather_status(ys=False) == 1
    assert gather_status(sigs=False) == 1
    assert gather_status(a=0) == 1
    assert gather_status(bias=0) == 1
    assert gather_status(flags=4) == 1
    assert gather_status(m=0) == 2
    assert gather_status(k=0) == 2
    assert gather_status(split=9) == 3
    assert gather_status(ldy=8000) == 5      # y_col_offset + N > row pitch
    assert gather_status(off=-1) == 5
    # 16-bit elements at odd addresses never reach a kernel
    assert gather_status(bias=17) == 1
    assert gather_status(a=17) == 1
    assert gather_status(b=17) == 1
    assert gather_status(ys_odd=True) == 1
    # valid arguments reach the device check: no sm_100a GPU here
    if not torch.cuda.is_available():
        assert gather_status() == 7


def test_gather_static_rejects_slots_outside_the_scratch():
    """The allocation-free gather takes its counter from a fixed array of
    GLQ_STATIC_GATHER_SLOTS words; other slots are refused before any device work."""
    lib = native.library()
    VP = ctypes.c_void_p
    ys = (VP * 1)(16)
    sigs = (VP * 1)(16)

    def call(slot):
        return lib.glq_linear_gather_static(0, 16, 4096, 1, 16, 1, 4096, 16, 2, ys, 4096, 0, 32, 4096, 4096, 0,
                                            0, 1, sigs, slot, 1, None, 0, None, None)
    scratch = native.STATUS_NAMES.index("scratch")
    assert call(-1) == scratch
    assert call(native.STATIC_GATHER_SLOTS) == scratch
    assert "static scratch" in native.status_string(scratch)
    if not torch.cuda.is_available():
        assert call(0) == 7
        assert call(native.STATIC_GATHER_SLOTS - 1) == 7


def test_gather_static_validates_before_touching_its_slot():
    """A call the library refuses (odd bias, bad rank, epoch 0) returns its
    status before the slot is cleared or the device is set up, so it cannot
    disturb another stream's call on the same slot."""
    lib = native.library()
    VP = ctypes.c_void_p
    ys = (VP * 1)(16)
    sigs = (VP * 1)(16)

    def call(bias=16, rank=0, epoch=1):
        return lib.glq_linear_gather_static(0, 16, 4096, 1, 16, 1, 4096, bias, 2, ys, 4096, 0, 32, 4096, 4096, 0,
                                            rank, 1, sigs, 0, epoch, None, 0, None, None)
    assert call(bias=17) == 1
    assert call(rank=1) == 1
    assert call(epoch=0) == 1


def raw_classes(base: int, rows: int, k: int, pitch: int):
    """Row classes of a raw-staged operand, as the library plans them: the
    smallest power of two C <= 8 with C * pitch a multiple of 8 elements and
    C * pitch >= k + 8; per class c the element offset s_c of its first row
    inside a 16-byte granule, and that granule's byte address."""
    pe = (k + 15) // 8 * 8 if rows <= 1 else pitch
    c = 1 if pe % 8 == 0 else 2 if pe % 4 == 0 else 4 if pe % 2 == 0 else 8
    while c < 8 and c * pe < k + 8:
        c *= 2
    if c * pe < k + 8:
        return None
    b0 = (base & 15) // 2
    classes = []
    for i in range(c):
        e = b0 + i * pe
        classes.append({"s": e & 7, "origin": (base & ~15) + 2 * (e - (e & 7)),
                        "rows": max(0, (rows - i + c - 1) // c)})
    return c, pe, classes


def raw_stage_image(mem: bytes, base: int, pitch: int, n_rows: int, k: int, k0: int, tile_rows: int = 128) -> bytes:
    """Host restatement of one stage of a raw-staged operand.

    TMA side: per row class c, one box of (tile_rows / C) rows x 72 elements
    at x = k0 of a map whose rows are class rows (pitch C * pitch elements,
    origin the granule below the class's first row), inner extent k + s_c,
    zero outside the map.  Shift side: chunk g of tile row r (class c = r % C,
    class row i = r / C) is raw granules g and g + 1 of that raw row, shifted
    by s_c elements, written at r * 128 + (g ^ (r % 8)) * 16.  The shift
    warps visit the rows in class order, four rows per warp step; every
    (row, chunk) is written once.  Class c's box lands c slots
    in, a slot being (tile_rows / C) * 144 bytes rounded up to 128.  `mem`
    holds the bytes at addresses 0 .. len(mem)."""
    c_count, pe, classes = raw_classes(base, n_rows, k, pitch)
    per = tile_rows // c_count
    # class c's box starts c slots in: per * 144 bytes rounded up to 128
    box = [c * (-(-per * 144 // 128) * 128) for c in range(c_count)]
    raw = bytearray(box[-1] + per * 144 + 32)
    for c, cl in enumerate(classes):
        for i in range(per):
            if i >= cl["rows"]:
                continue
            for x in range(k0, k0 + 72):
                if x < k + cl["s"]:
                    addr = cl["origin"] + 2 * (i * c_count * pe + x)
                    off = box[c] + i * 144 + 2 * (x - k0)
                    raw[off:off + 2] = mem[addr:addr + 2]
    stage = bytearray(tile_rows * 128)
    written = set()
    log_c = c_count.bit_length() - 1
    rpc = tile_rows // c_count
    for u in range(tile_rows // 4):  # warp steps (contiguous blocks per shift warp)
        for lane in range(32):
            idx = 4 * u + lane // 8
            g = lane % 8
            c, i = idx // rpc, idx % rpc
            r = (i << log_c) + c
            s = classes[c]["s"]
            row = box[c] + i * 144 + 16 * g
            window = bytes(raw[row: row + 32])
            off = r * 128 + ((g ^ (r % 8)) * 16)
            stage[off:off + 16] = window[2 * s: 2 * s + 16]
            written.add((r, g))
    assert len(written) == tile_rows * 8
    return bytes(stage)


@pytest.mark.parametrize("k,pitch,base,rows", [(4090, 4090, 64, 100), (4096, 4098, 128, 100), (4096, 4096, 130, 100),
                                               (1001, 1001, 70, 100), (131, 135, 2, 100), (4096, 4096, 2, 1),
                                               (4090, 4090, 6, 32), (200, 201, 14, 3), (1001, 1001, 2, 16)])
def test_raw_stage_restatement(k, pitch, base, rows):
    """Row-class boxes plus the in-shared-memory shift give exactly the
    128-byte-swizzled K-major tile of the rows: what a TMA load with zero
    fill writes from an aligned copy (rows >= N and columns >= K zero)."""
    rng = np.random.default_rng(k + pitch + base + rows)
    mem = rng.integers(0, 256, size=base + rows * pitch * 2 + 64, dtype=np.uint8).tobytes()
    tile_rows = 128 if rows > 32 else 32 if rows > 16 else 16
    for k0 in range(0, k, 64 * max(1, k // 256)):
        got = raw_stage_image(mem, base, pitch, rows, k, k0, tile_rows)
        want = bytearray(tile_rows * 128)
        for r in range(min(rows, tile_rows)):
            row = mem[base + r * pitch * 2 + 2 * k0: base + r * pitch * 2 + 2 * min(k, k0 + 64)]
            dense = row + bytes(128 - len(row))
            for off in range(0, 128, 16):
                linear = r * 128 + off
                swz = linear ^ (((linear >> 7) & 7) << 4)  # 128-byte swizzle: bits 4-6 ^= bits 7-9
                want[swz:swz + 16] = dense[off:off + 16]
        assert got == bytes(want), f"k0={k0}"


def test_raw_class_maps_stay_inside_the_operand():
    """Every byte a class map can read (its rows x (k + s_c) elements from its
    origin) lies inside the 16-byte granules that hold the operand's rows,
    and the class rows do not overlap."""
    for base, rows, k, pitch in [(2, 4096, 4090, 4090), (66, 33, 1001, 1003), (130, 7, 4096, 4096),
                                 (14, 1, 77, 77), (6, 100, 131, 135)]:
        c_count, pe, classes = raw_classes(base, rows, k, pitch)
        assert (c_count * pe) % 8 == 0 and c_count * pe >= k + 8
        first = base & ~15
        last = (base + 2 * ((rows - 1) * pitch + k) + 15) & ~15
        for c, cl in enumerate(classes):
            assert cl["origin"] % 16 == 0
            if cl["rows"]:
                lo = cl["origin"]
                hi = cl["origin"] + 2 * ((cl["rows"] - 1) * c_count * pe + k + cl["s"])
                assert first <= lo and hi <= last
                # row i of the class starts at the class row's element s_c
                for i in range(cl["rows"]):
                    r = c + c_count * i
                    assert cl["origin"] + 2 * (i * c_count * pe + cl["s"]) == base + 2 * r * pitch
