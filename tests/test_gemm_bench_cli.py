"""The native gemm_bench CLI: the lab's flags, JSON schema v1 and exit codes.

Ports the reference's CTest matrix (CMakeLists.txt:34-90): every edge shape
through each tensor-core implementation, FP16 and BF16, one sample each; the
CLI checks the output against cuBLAS element by element before timing and
exits 1 on a failed gate.  The CPU tests cover --help and the rejections,
which run before any CUDA call.
"""
from __future__ import annotations

import json
import subprocess

import pytest

from gemm_lab_qualification_b200 import build

EDGE_SHAPES = ["17x31x13", "129x257x65", "127x129x131", "1x4096x4096", "509x4099x4103", "256x256x256"]
OUR_IMPLS = ["glq", "glq_splitk", "glq_wnk"]


@pytest.fixture(scope="module")
def cli() -> str:
    return str(build.build_bench())


def run(cli: str, *args: str, timeout: int = 180) -> subprocess.CompletedProcess:
    return subprocess.run([cli, *args], capture_output=True, text=True, timeout=timeout)


def test_help_lists_the_implementations(cli):
    out = run(cli, "--help")
    assert out.returncode == 0
    for name in ["cublas", "cublaslt", *OUR_IMPLS, "--cache steady|cold", "--split-k"]:
        assert name in out.stdout


@pytest.mark.parametrize("args,message", [
    (["--impl", "wmma"], "--impl must be"),
    (["--impl", "glq", "--dtype", "fp32"], "fp16 or bf16"),
    (["--dtype", "fp8"], "--dtype must be"),
    (["--cache", "warm"], "--cache must be"),
    (["--m", "-3"], "--m needs an integer"),
    (["--split-k", "9"], "--split-k needs an integer in 0..8"),
    (["--samples", "0"], "--samples must be positive"),
    (["--bogus", "1"], "unknown option"),
    (["--m"], "no value after --m"),
])
def test_rejections_exit_1(cli, args, message):
    out = run(cli, *args)
    assert out.returncode == 1
    assert message in out.stderr


def check_json(stdout: str) -> dict:
    doc = json.loads(stdout)
    assert doc["schema_version"] == 1
    assert doc["correctness"]["passed"] is True
    assert doc["benchmark"]["samples"] >= 1
    assert doc["benchmark"]["latency_ms"]["p50"] > 0
    return doc


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("impl", OUR_IMPLS)
@pytest.mark.parametrize("shape", EDGE_SHAPES)
def test_ctest_matrix(cli, cuda_device, shape, impl, dtype):
    m, n, k = shape.split("x")
    out = run(cli, "--m", m, "--n", n, "--k", k, "--dtype", dtype, "--impl", impl, "--warmup", "0",
              "--samples", "1", "--measurement-seconds", "0")
    assert out.returncode == 0, out.stderr
    doc = check_json(out.stdout)
    assert doc["correctness"]["reference"] == "cublas_full"
    assert doc["correctness"]["elements_checked"] == int(m) * int(n)
    assert doc["implementation"]["path"]


@pytest.mark.gpu
def test_vendor_references_and_cold_cache(cli, cuda_device):
    for impl in ["cublas", "cublaslt"]:
        out = run(cli, "--m", "32", "--n", "4096", "--k", "4096", "--impl", impl, "--samples", "3")
        assert out.returncode == 0, out.stderr
        assert check_json(out.stdout)["correctness"]["reference"] == "cpu_fp64_spot"
    out = run(cli, "--m", "32", "--n", "4096", "--k", "4096", "--impl", "glq_splitk", "--split-k", "4",
              "--cache", "cold", "--samples", "5", "--pretty")
    assert out.returncode == 0, out.stderr
    doc = check_json(out.stdout)
    assert doc["benchmark"]["cache_mode"] == "cold"
    assert doc["benchmark"]["split_k"] == 4
    assert doc["benchmark"]["workspace_bytes"] == 4 * 32 * 4096 * 4
    assert doc["implementation"]["path"] == "tc_kn"
