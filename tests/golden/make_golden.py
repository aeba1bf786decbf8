"""Generate the golden fixtures of tests/golden/ from the reference itself.

Run in a checkout where the reference project is importable:

    python tests/golden/make_golden.py --reference /path/to/gemm-lab-qualification

It imports the reference's own ``qualification`` module (CPU only) and records
what ``qualification.reference`` (FP64 matmul + 64-dot fsum cross-check,
qualification.py:24-31) returns on:

* the reference manifest's edge corpus (5 shapes x 3 patterns,
  manifests/workloads.json:14-20) with ``qualification.inputs``, plus the
  fused epilogue target ``silu(expected + linspace(-.2, .2, n))``
  (qualification.py:95-98);
* the manifest's benchmark shapes (decode-m8, decode-m32, tail, square):
  full tensors for the small ones, input sha256 + selected output rows for
  the 4096-wide ones;
* the known-answer 2x2 of tests/test_contract.py:36-44;
* the seed-7 uniform contract of this build (A, W [N, K], bias drawn in that
  order) at M in {1, 8, 32, 128}, N = K = 4096: input sha256, full output
  for M = 1, rows 0 and M-1 otherwise, for both the plain GEMM and the fused
  bias + SiLU target; and one small uniform case stored whole.

The outputs are ``corpus.npz`` (arrays) and ``manifest.json`` (hashes,
shapes, provenance).  Nothing at test time reads the reference.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def sha(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="root of the reference project")
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    import qualification as q  # the reference's own module

    sys.path.insert(0, str(REPO))
    from gemm_lab_qualification_b200.workloads import uniform_inputs

    arrays: dict[str, np.ndarray] = {}
    meta: dict = {"generator": "tests/golden/make_golden.py",
                  "reference_module": "qualification.py (reference project)",
                  "reference_seed": q.MANIFEST["seed"], "cases": {}}

    # Edge corpus: every shape x pattern; layouts share values.
    for shape in q.MANIFEST["edges"]:
        for pattern in q.MANIFEST["edge_patterns"]:
            a, b = q.inputs(shape, pattern, "contiguous")
            expected = q.reference(a, b)
            key = f"edge/{shape['id']}/{pattern}"
            arrays[key + "/a"] = u16(a)
            arrays[key + "/b"] = u16(b)
            arrays[key + "/expected"] = expected.numpy()
            if shape["m"] and shape["n"]:
                bias = torch.linspace(-.2, .2, shape["n"], dtype=torch.float16)
                fused = torch.nn.functional.silu(expected + bias.double())
                arrays[key + "/fused"] = fused.numpy()
            meta["cases"][key] = {"m": shape["m"], "n": shape["n"], "k": shape["k"], "full": True}

    # Manifest benchmark shapes.
    for shape in q.MANIFEST["benchmark"]:
        a, b = q.inputs(shape, "random", "contiguous")
        expected = q.reference(a, b)
        key = f"bench/{shape['id']}"
        m, n = shape["m"], shape["n"]
        bias = torch.linspace(-.2, .2, n, dtype=torch.float16)
        fused = torch.nn.functional.silu(expected + bias.double())
        entry = {"m": m, "n": n, "k": shape["k"], "input_sha256": sha(a, b)}
        if a.numel() + b.numel() <= 1 << 16:
            arrays[key + "/a"] = u16(a)
            arrays[key + "/b"] = u16(b)
            arrays[key + "/expected"] = expected.numpy()
            arrays[key + "/fused"] = fused.numpy()
            entry["full"] = True
        else:
            rows = sorted({0, m - 1})
            arrays[key + "/rows"] = np.array(rows, dtype=np.int64)
            arrays[key + "/expected_rows"] = expected[rows].numpy()
            arrays[key + "/fused_rows"] = fused[rows].numpy()
            entry["full"] = False
            entry["rows"] = rows
        meta["cases"][key] = entry

    # Known-answer test (tests/test_contract.py:36-44).
    a = torch.tensor([[1., -2.], [3., 4.]], dtype=torch.float16)
    b = torch.tensor([[2., 5.], [-1., 6.]], dtype=torch.float16)
    arrays["kat/a"] = u16(a)
    arrays["kat/b"] = u16(b)
    arrays["kat/expected"] = q.reference(a, b).numpy()
    meta["cases"]["kat"] = {"m": 2, "n": 2, "k": 2, "full": True}

    # Seed-7 uniform contract (the headline configs), reference oracle on our inputs.
    for m in (1, 8, 32, 128):
        n = k = 4096
        a, w, bias = uniform_inputs(m, n, k)
        expected = q.reference(a, w.t())
        fused = torch.nn.functional.silu(expected + bias.double())
        key = f"uniform/m{m}"
        rows = list(range(m)) if m == 1 else sorted({0, m - 1})
        arrays[key + "/rows"] = np.array(rows, dtype=np.int64)
        arrays[key + "/expected_rows"] = expected[rows].numpy()
        arrays[key + "/fused_rows"] = fused[rows].numpy()
        meta["cases"][key] = {"m": m, "n": n, "k": k, "full": False, "rows": rows,
                              "a_sha256": sha(a), "w_sha256": sha(w), "bias_sha256": sha(bias)}

    m, n, k = 8, 256, 512
    a, w, bias = uniform_inputs(m, n, k)
    expected = q.reference(a, w.t())
    key = "uniform/small"
    arrays[key + "/a"] = u16(a)
    arrays[key + "/w"] = u16(w)
    arrays[key + "/bias"] = u16(bias)
    arrays[key + "/expected"] = expected.numpy()
    arrays[key + "/fused"] = torch.nn.functional.silu(expected + bias.double()).numpy()
    meta["cases"][key] = {"m": m, "n": n, "k": k, "full": True}

    np.savez_compressed(HERE / "corpus.npz", **arrays)
    (HERE / "manifest.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(arrays)} arrays, {len(meta['cases'])} cases")
    return 0


if __name__ == "__main__":
    sys.exit(main())
