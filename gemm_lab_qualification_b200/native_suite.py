"""Native suite: the gemm_bench CLI run as one process per measurement.

Follows native_suite.py:5-19 of the reference:

* every ``benchmark`` shape of the workload manifest x each implementation,
  in 3 rounds whose order is reshuffled by ``random.Random(1729)``;
* each child is ``gemm_bench --m --n --k --dtype fp16 --impl I --warmup 10
  --samples 31 --measurement-seconds 0 --seed 1729``, validates its output
  against cuBLAS before warm-up and timing, and prints one JSON record;
* a child that exits non-zero, or whose record says the correctness gate
  failed, aborts the suite (RuntimeError / AssertionError, as there).

The reference times its sm_89 ladder (cublaslt, ptx_mma_small,
ptx_mma_splitk); here the rows are cuBLASLt and this library's sm_100a
implementations (``glq`` = planned path on B[K, N], ``glq_splitk`` = split-K
with the FP32 partial workspace, ``glq_wnk`` = K-contiguous weight).  The
reference suite measures the steady (warm-L2) cache mode only
(native_suite.py:11-12); this one also runs ``--cache cold`` (L2 overwritten
before each sample), which is the mode the HBM roofline fraction refers to.

``python -m gemm_lab_qualification_b200.native_suite --output suite.json``;
``summarize.py`` renders the result as Markdown.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import platform
import random
import subprocess
import sys
import tempfile
from datetime import datetime, timezone
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
MANIFEST = json.loads((PACKAGE_DIR / "workloads.json").read_text())
IMPLS = ("cublaslt", "glq", "glq_splitk", "glq_wnk")
CACHE_MODES = ("steady", "cold")
SEED = 1729
ROUNDS = 3
PROTOCOL = ("3 shuffled rounds; one gemm_bench process per measurement; each child validates against cuBLAS "
            "before warm-up and timing; no sanitizer or profiler in the timed process; cold = L2 overwritten "
            "and the stream synchronised before each single-call sample")


def source_digest() -> str:
    """SHA-256 over the library and CLI sources (csrc, include, manifest)."""
    h = hashlib.sha256()
    files = sorted((PACKAGE_DIR / "csrc").glob("*")) + sorted((PACKAGE_DIR.parent / "include").glob("*.h"))
    for path in [*files, PACKAGE_DIR / "workloads.json"]:
        if path.is_file():
            h.update(path.name.encode())
            h.update(path.read_bytes())
    return h.hexdigest()


def _command(args: list[str]) -> dict:
    try:
        p = subprocess.run(args, capture_output=True, text=True, timeout=60)
        return {"returncode": p.returncode, "stdout": p.stdout}
    except (OSError, subprocess.TimeoutExpired) as e:
        return {"returncode": None, "error": str(e)}


def environment() -> dict:
    """Host, GPU and toolchain identity of a suite run (read-only queries)."""
    return {"utc": datetime.now(timezone.utc).isoformat(), "python": sys.version, "platform": platform.platform(),
            "source_digest": source_digest(),
            "gpu": _command(["nvidia-smi", "--query-gpu=name,uuid,driver_version,compute_cap,clocks.sm,clocks.max.sm,"
                             "power.draw,power.limit,memory.total", "--format=csv"]),
            "nvcc": _command(["nvcc", "--version"]),
            "measurement_policy": {"clock_changes": False, "scope": "one GPU; unlocked clocks"}}


def require_gate(path: str | os.PathLike) -> dict:
    """A correctness gate must have passed on the same sources (evidence.py:71-74)."""
    gate = json.loads(Path(path).read_text())
    if gate.get("status") != "passed" or gate.get("environment", {}).get("source_digest") != source_digest():
        raise RuntimeError("missing, failed, or stale correctness gate")
    return gate


def save(path: str | os.PathLike, data: dict) -> None:
    """Serialise first, then replace the target atomically (evidence.py:48-60)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    payload = json.dumps(data, indent=2, sort_keys=True, allow_nan=False) + "\n"
    fd, tmp = tempfile.mkstemp(prefix="." + path.name + ".", suffix=".tmp", dir=path.parent)
    try:
        with os.fdopen(fd, "w") as stream:
            stream.write(payload)
            stream.flush()
            os.fsync(stream.fileno())
        os.replace(tmp, path)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)


def child_args(binary: str | os.PathLike, shape: dict, impl: str, cache: str, warmup: int = 10,
               samples: int = 31) -> list[str]:
    return [str(binary), "--m", str(shape["m"]), "--n", str(shape["n"]), "--k", str(shape["k"]), "--dtype", "fp16",
            "--impl", impl, "--cache", cache, "--warmup", str(warmup), "--samples", str(samples),
            "--measurement-seconds", "0", "--seed", str(SEED)]


def run(gate: str | os.PathLike | None = None, binary: str | os.PathLike | None = None,
        shapes: list[dict] | None = None, impls: tuple[str, ...] = IMPLS,
        cache_modes: tuple[str, ...] = CACHE_MODES, rounds: int = ROUNDS, warmup: int = 10,
        samples: int = 31, timeout: float = 120.0) -> dict:
    """Run the suite; returns the evidence document (``results`` = one row per child)."""
    gate_doc = require_gate(gate) if gate is not None else None
    if binary is None:
        from . import build
        binary = build.build_bench()
    binary = Path(binary)
    shapes = list(MANIFEST["benchmark"]) if shapes is None else shapes
    rng = random.Random(SEED)
    tasks = [(s, impl, cache) for s in shapes for impl in impls for cache in cache_modes]
    rows = []
    for round_id in range(rounds):
        rng.shuffle(tasks)
        for shape, impl, cache in tasks:
            args = child_args(binary, shape, impl, cache, warmup, samples)
            p = subprocess.run(args, text=True, capture_output=True, timeout=timeout)
            if p.returncode:
                raise RuntimeError(f"{' '.join(args[1:])}: exit {p.returncode}: {p.stderr.strip()}")
            record = json.loads(p.stdout)
            if not record["correctness"]["passed"]:
                raise AssertionError(f"native correctness failed: {shape['id']} {impl} {cache}")
            rows.append({"round": round_id, "case": shape["id"], "cache": cache, "argv": args, "record": record,
                         "stderr": p.stderr})
    return {"status": "measured", "environment": environment(),
            "binary_sha256": hashlib.sha256(binary.read_bytes()).hexdigest(), "seed": SEED,
            "gate": None if gate_doc is None else str(gate), "results": rows, "protocol": PROTOCOL}


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gate", help="correctness gate JSON that must have passed on these sources")
    p.add_argument("--output", required=True)
    p.add_argument("--binary", help="gemm_bench path (default: build it in-tree)")
    p.add_argument("--rounds", type=int, default=ROUNDS)
    p.add_argument("--impls", default=",".join(IMPLS))
    p.add_argument("--cache", default=",".join(CACHE_MODES))
    a = p.parse_args(argv)
    save(a.output, run(a.gate, a.binary, impls=tuple(a.impls.split(",")), cache_modes=tuple(a.cache.split(",")),
                       rounds=a.rounds))
    return 0


if __name__ == "__main__":
    sys.exit(main())
