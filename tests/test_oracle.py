"""The CPU oracle, pinned against the reference's own outputs (CPU only).

Golden vectors come from ``tests/golden/make_golden.py``, which ran the
reference's ``qualification.reference`` on these inputs.  The oracle is a
separate FP64 implementation (numpy, different summation order), so it must
agree to FP64 rounding, not bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import f16
from gemm_lab_qualification_b200 import workloads
from oracle import reference as oracle

PIN = 1e-9  # |oracle - golden| <= PIN * max(1, |golden|)


def assert_pinned(actual: np.ndarray, golden: np.ndarray) -> None:
    assert actual.shape == golden.shape
    bound = PIN * np.maximum(1.0, np.abs(golden))
    assert (np.abs(actual - golden) <= bound).all()


def edge_keys(manifest):
    return sorted(k for k in manifest["cases"] if k.startswith("edge/"))


def test_edge_corpus_matches_reference(golden):
    arrays, manifest = golden
    keys = edge_keys(manifest)
    assert len(keys) == 15  # 5 shapes x 3 patterns
    for key in keys:
        a = f16(arrays[key + "/a"])
        b = f16(arrays[key + "/b"])
        out = oracle.reference(a, b)
        assert_pinned(out, arrays[key + "/expected"])
        if key + "/fused" in arrays:
            # bias = linspace(-.2, .2, n) in FP16 (qualification.py:95)
            n = b.shape[1]
            bias = torch.linspace(-.2, .2, n, dtype=torch.float16).numpy()
            assert_pinned(oracle.silu_reference(out, bias), arrays[key + "/fused"])


def test_generator_reproduces_reference_inputs(golden):
    arrays, manifest = golden
    for key in edge_keys(manifest):
        _, sid, pattern = key.split("/")
        shape = next(s for s in workloads.MANIFEST["edges"] if s["id"] == sid)
        a, b = workloads.inputs(shape, pattern, "contiguous")
        assert np.array_equal(a.view(torch.int16).numpy().view(np.uint16), arrays[key + "/a"])
        assert np.array_equal(b.view(torch.int16).numpy().view(np.uint16), arrays[key + "/b"])


def test_known_answer(golden):
    arrays, _ = golden
    out = oracle.reference(f16(arrays["kat/a"]), f16(arrays["kat/b"]))
    assert np.array_equal(out, np.array([[4., -7.], [2., 39.]]))
    assert np.array_equal(out, arrays["kat/expected"])


def test_benchmark_shapes(golden):
    arrays, manifest = golden
    for shape in workloads.MANIFEST["benchmark"]:
        key = f"bench/{shape['id']}"
        case = manifest["cases"][key]
        a, b = workloads.inputs(shape)
        assert workloads.sha256_of(a, b) == case["input_sha256"]
        if case["full"]:
            out = oracle.reference(a, b)
            assert_pinned(out, arrays[key + "/expected"])
        else:
            rows = arrays[key + "/rows"]
            out = oracle.reference(a[rows], b, samples=8)
            assert_pinned(out, arrays[key + "/expected_rows"])
            bias = workloads.reference_bias(shape["n"]).numpy()
            assert_pinned(oracle.silu_reference(out, bias), arrays[key + "/fused_rows"])


@pytest.mark.parametrize("m", [1, 8, 32, 128])
def test_uniform_contract_inputs_and_rows(golden, m):
    arrays, manifest = golden
    key = f"uniform/m{m}"
    case = manifest["cases"][key]
    a, w, bias = workloads.uniform_inputs(m, 4096, 4096)
    assert workloads.sha256_of(a) == case["a_sha256"]
    assert workloads.sha256_of(w) == case["w_sha256"]
    assert workloads.sha256_of(bias) == case["bias_sha256"]
    assert float(a.float().min()) >= -0.5 and float(a.float().max()) <= 0.5
    rows = arrays[key + "/rows"]
    out = oracle.linear_reference(a[rows], w, samples=8)
    assert_pinned(out, arrays[key + "/expected_rows"])
    fused = oracle.linear_reference(a[rows], w, bias, silu=True, samples=8)
    assert_pinned(fused, arrays[key + "/fused_rows"])


def test_uniform_small_full(golden):
    arrays, _ = golden
    a = f16(arrays["uniform/small/a"])
    w = f16(arrays["uniform/small/w"])
    bias = f16(arrays["uniform/small/bias"])
    assert_pinned(oracle.linear_reference(a, w), arrays["uniform/small/expected"])
    assert_pinned(oracle.linear_reference(a, w, bias, silu=True), arrays["uniform/small/fused"])
    ta, tw, tb = workloads.uniform_inputs(8, 256, 512)
    assert np.array_equal(ta.numpy(), a) and np.array_equal(tw.numpy(), w) and np.array_equal(tb.numpy(), bias)


@pytest.mark.parametrize("mutation", ["transpose", "tail", "nan", "scale"])
def test_detector_mutations(golden, mutation):
    """compare() must reject corrupted outputs (tests/test_contract.py:16-23)."""
    arrays, _ = golden
    r = arrays["edge/odd/random/expected"]
    bad = r.copy()
    if mutation == "transpose":
        bad = bad.T
    if mutation == "tail":
        bad[-1, -1] += 1
    if mutation == "nan":
        bad[0, 0] = float("nan")
    if mutation == "scale":
        bad *= 2
    with pytest.raises(AssertionError):
        oracle.compare(bad, r)


@pytest.mark.parametrize("value", [float("nan"), float("inf"), -float("inf"), 65504.])
def test_invalid_numerics(value):
    """Input qualification (tests/test_contract.py:25-28)."""
    a = np.full((1, 1), value, dtype=np.float16)
    b = np.full((1, 1), 2., dtype=np.float16)
    with pytest.raises(ValueError):
        oracle.reference(a, b)


def test_crosscheck_rejects_corrupt_reference():
    a = np.array([[1., -2.], [3., 4.]], dtype=np.float16)
    b = np.array([[2., 5.], [-1., 6.]], dtype=np.float16)
    expected = a.astype(np.float64) @ b.astype(np.float64)
    oracle.crosscheck_reference(a, b, expected)
    expected[-1, -1] += 1
    with pytest.raises(AssertionError, match="scalar reference mismatch"):
        oracle.crosscheck_reference(a, b, expected)


def test_uniform_gate_bounds():
    """The uniform-corpus gate: pass at the bound, fail just beyond it."""
    expected = np.array([[10.0, -3.0]])
    ok = expected + np.array([[0.02 + 0.002 * 10.0, -(0.02 + 0.002 * 3.0)]]) * 0.999
    oracle.compare(ok, expected, oracle.UNIFORM_ATOL, oracle.UNIFORM_RTOL)
    bad = expected + np.array([[0.02 + 0.002 * 10.0, 0.0]]) * 1.01
    with pytest.raises(AssertionError):
        oracle.compare(bad, expected, oracle.UNIFORM_ATOL, oracle.UNIFORM_RTOL)


@pytest.mark.parametrize("k,splits,granule", [(4096, 4, 64), (4090, 8, 64), (131, 2, 64), (4096, 8, 8),
                                              (4093, 3, 8), (13, 2, 8)])
def test_split_ranges_partition_k(k, splits, granule):
    ranges = oracle.split_ranges(k, splits, granule)
    assert ranges[0][0] == 0 and ranges[-1][1] == k
    for (lo0, hi0), (lo1, _) in zip(ranges, ranges[1:]):
        assert hi0 == lo1 and lo0 <= hi0
    a = np.random.default_rng(0).standard_normal((3, k)).astype(np.float16)
    b = np.random.default_rng(1).standard_normal((k, 5)).astype(np.float16)
    parts = oracle.split_partials_reference(a, b, splits, granule)
    full = a.astype(np.float64) @ b.astype(np.float64)
    assert np.allclose(parts.sum(axis=0), full, rtol=0, atol=1e-9 * max(1.0, float(np.abs(full).max())))
