"""CPU oracle of the FP16 linear (+ bias + SiLU) path -- TEST INFRASTRUCTURE.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it.  The shipped operators (``gemm_lab_qualification_b200``) never
call it and have no CPU path.

It restates, in numpy FP64, the reference lab's qualification contract
(paths inside the reference project):

* ``reference``            -- qualification.py:24-31: input qualification
  (rank, FP16, finite), FP64 ``A @ B``, the scalar cross-check, and the
  FP16 output-overflow exclusion.
* ``crosscheck_reference`` -- qualification.py:33-45: ``samples`` evenly
  spread dot products recomputed with ``math.fsum`` (exactly rounded) and
  compared at rel 1e-12 / abs 1e-10.
* ``compare``              -- qualification.py:47-56: the tolerance gate
  ``|actual - expected| <= atol + rtol * |expected|`` with every output
  finite, returning max_abs / max_scaled_error / rms.
* ``silu_reference``       -- the fused epilogue's FP64 reference,
  ``silu(expected + bias)`` (qualification.py:95-98; the kernel it checks is
  kernels.py:244-246).
* ``split_ranges``         -- the K ranges of a split-K call, to check the
  per-split FP32 partials the kernels write (the reference's partial
  layout [S, M, N], kernels.py:431-439).

Parity is pinned: ``tests/test_oracle.py`` checks this module against the
golden vectors that ``tests/golden/make_golden.py`` produced by running the
reference's own ``qualification.reference`` on the same inputs.
"""
from __future__ import annotations

import math

import numpy as np

# Gate for the seed-7 uniform corpus: abs <= 0.02 + 0.002 * |ref|.
UNIFORM_ATOL = 0.02
UNIFORM_RTOL = 0.002
# The reference corpus' own gates (manifests/workloads.json:6-7,
# qualification.py:98).
REFERENCE_ATOL = 0.003
REFERENCE_RTOL = 0.005
FUSED_ATOL = 0.01
FUSED_RTOL = 0.01
FP16_MAX = 65504.0


def _as_numpy(x) -> np.ndarray:
    """Accept numpy arrays or CPU/GPU torch tensors (converted, not shared)."""
    if isinstance(x, np.ndarray):
        return x
    # torch tensor: bfloat16 has no numpy dtype, widen losslessly first.
    t = x.detach().cpu()
    if str(t.dtype) == "torch.bfloat16":
        t = t.float()
    return t.numpy()


def reference(a, b, samples: int = 64, check_dtype: bool = True) -> np.ndarray:
    """FP64 A @ B with the reference's input qualification and cross-check.

    a: [M, K], b: [K, N], both FP16 (qualification.py:26).  Returns a float64
    [M, N] array.  Raises ValueError on a contract violation and
    AssertionError when the scalar cross-check disagrees.
    """
    a = _as_numpy(a)
    b = _as_numpy(b)
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("shape contract")
    if check_dtype and (a.dtype != np.float16 or b.dtype != a.dtype):
        raise ValueError("v1 is FP16 only")
    a64 = a.astype(np.float64)
    b64 = b.astype(np.float64)
    if not np.isfinite(a64).all() or not np.isfinite(b64).all():
        raise ValueError("finite input contract")
    out = a64 @ b64
    crosscheck_reference(a64, b64, out, samples=samples)
    if (np.abs(out) > FP16_MAX).any():
        raise ValueError("FP16 output overflow excluded")
    return out


def crosscheck_reference(a, b, expected, samples: int = 64) -> None:
    """Recompute ``samples`` dots with math.fsum at evenly spread indices.

    Indices (j * (m*n - 1)) // (count - 1) include both corners
    (qualification.py:38-40).  Every product of two FP16 values is exact in
    FP64, so fsum gives the exactly rounded dot product.
    """
    a = np.asarray(_as_numpy(a), dtype=np.float64)
    b = np.asarray(_as_numpy(b), dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    m, k = a.shape
    n = b.shape[1]
    if not m or not n:
        return
    count = min(samples, m * n)
    indices = [0] if count == 1 else [(j * (m * n - 1)) // (count - 1) for j in range(count)]
    for index in indices:
        row, col = divmod(index, n)
        scalar = math.fsum((a[row, :] * b[:, col]).tolist())
        if not math.isclose(float(expected[row, col]), scalar, rel_tol=1e-12, abs_tol=1e-10):
            raise AssertionError(f"independent scalar reference mismatch at ({row},{col})")


def compare(actual, expected, atol: float = REFERENCE_ATOL, rtol: float = REFERENCE_RTOL) -> dict:
    """The tolerance gate (qualification.py:47-56)."""
    actual = np.asarray(_as_numpy(actual), dtype=np.float64)
    expected = np.asarray(_as_numpy(expected), dtype=np.float64)
    if actual.shape != expected.shape:
        raise AssertionError("output shape mismatch")
    error = np.abs(actual - expected)
    bound = atol + rtol * np.abs(expected)
    if not np.isfinite(actual).all() or not (error <= bound).all():
        worst = float(np.nanmax(error)) if error.size else 0.0
        raise AssertionError(f"numerical gate: max absolute error {worst}")
    if not error.size:
        return {"max_abs": 0.0, "max_scaled_error": 0.0, "rms": 0.0}
    return {"max_abs": float(error.max()), "max_scaled_error": float((error / bound).max()),
            "rms": float(np.sqrt(np.mean(np.square(error))))}


def silu_reference(expected, bias) -> np.ndarray:
    """FP64 silu(expected + bias[None, :]) = v / (1 + exp(-v))."""
    expected = np.asarray(expected, dtype=np.float64)
    bias = np.asarray(_as_numpy(bias), dtype=np.float64)
    v = expected + bias[None, :]
    with np.errstate(over="ignore"):
        return v / (1.0 + np.exp(-v))


def linear_reference(a, w, bias=None, silu: bool = False, samples: int = 64) -> np.ndarray:
    """FP64 y = [silu](a @ w.T [+ bias]) for a linear weight w [N, K]."""
    w = _as_numpy(w)
    out = reference(a, w.T, samples=samples, check_dtype=False)
    if bias is None:
        return out
    if silu:
        return silu_reference(out, bias)
    return out + np.asarray(_as_numpy(bias), dtype=np.float64)[None, :]


def split_ranges(k: int, splits: int, granule: int) -> list[tuple[int, int]]:
    """K ranges [lo, hi) of each split: ``granule``-wide blocks divided as
    blocks*s//S .. blocks*(s+1)//S (64 for the tcgen05 kernel, 8 for the
    GEMV; the GEMV's K % 8 remainder belongs to the last split)."""
    blocks = (k + granule - 1) // granule if granule == 64 else k // granule
    out = []
    for s in range(splits):
        lo = (blocks * s) // splits * granule
        hi = (blocks * (s + 1)) // splits * granule
        if s == splits - 1:
            hi = k
        out.append((min(lo, k), min(hi, k)))
    return out


def split_partials_reference(a, b, splits: int, granule: int) -> np.ndarray:
    """FP64 per-split partial sums [S, M, N] of A @ B over split_ranges."""
    a64 = np.asarray(_as_numpy(a), dtype=np.float64)
    b64 = np.asarray(_as_numpy(b), dtype=np.float64)
    out = np.zeros((splits, a64.shape[0], b64.shape[1]))
    for s, (lo, hi) in enumerate(split_ranges(a64.shape[1], splits, granule)):
        out[s] = a64[:, lo:hi] @ b64[lo:hi, :]
    return out
