"""Deterministic inputs of the qualification contract.

Two generators, both on the CPU torch generator so the bytes are identical on
every machine (the committed fixtures pin them by sha256):

* ``uniform_inputs`` -- the seed-7 contract: FP32 draws uniform in
  [-0.5, 0.5) from ``torch.Generator().manual_seed(7)`` in the order A, W,
  bias, rounded to FP16 (or BF16).  W is [N, K] row-major (K-contiguous).
* ``inputs`` -- the reference lab's own corpus generator
  (qualification.py:9-22): seed 1729, ``randn * 0.2``, B = [K, N], the
  ``zeros`` / ``cancellation`` patterns and the NaN-poisoned ``strided``
  layout.

Plus the probe layouts of the boundary corpus (padded rows, transposed A,
misaligned base) built inside poisoned storage.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

MANIFEST = json.loads((Path(__file__).resolve().parent / "workloads.json").read_text())


def uniform_inputs(m: int, n: int, k: int, seed: int | None = None,
                   dtype: torch.dtype = torch.float16) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(A [m, k], W [n, k], bias [n]) on the CPU, draws in the order A, W, bias."""
    contract = MANIFEST["uniform_contract"]
    g = torch.Generator().manual_seed(contract["seed"] if seed is None else seed)
    lo, hi = contract["low"], contract["high"]
    a = torch.empty((m, k), dtype=torch.float32).uniform_(lo, hi, generator=g).to(dtype)
    w = torch.empty((n, k), dtype=torch.float32).uniform_(lo, hi, generator=g).to(dtype)
    bias = torch.empty((n,), dtype=torch.float32).uniform_(lo, hi, generator=g).to(dtype)
    return a, w, bias


def inputs(shape: dict, pattern: str = "random", layout: str = "contiguous") -> tuple[torch.Tensor, torch.Tensor]:
    """The reference corpus generator (qualification.py:9-22), B = [K, N]."""
    m, n, k = (shape[x] for x in ("m", "n", "k"))
    g = torch.Generator().manual_seed(MANIFEST["reference_contract"]["seed"])
    a = (torch.randn((m, k), generator=g) * .2).half()
    b = (torch.randn((k, n), generator=g) * .2).half()
    if pattern == "zeros":
        a.zero_()
        b.zero_()
    elif pattern == "cancellation":
        a.fill_(256)
        b.fill_(.125)
        b[1::2].neg_()
    elif pattern != "random":
        raise ValueError(pattern)
    if layout == "strided":
        aa = torch.full((m, k * 2 + 2), float("nan"), dtype=a.dtype)
        aa[:, 1:1 + 2 * k:2] = a
        a = aa[:, 1:1 + 2 * k:2]
        bb = torch.full((k, n * 2 + 2), float("nan"), dtype=b.dtype)
        bb[:, 1:1 + 2 * n:2] = b
        b = bb[:, 1:1 + 2 * n:2]
    elif layout != "contiguous":
        raise ValueError(layout)
    return a, b


def reference_bias(n: int, dtype: torch.dtype = torch.float16, device: str | torch.device = "cpu") -> torch.Tensor:
    """Bias of the reference corpus' fused check (qualification.py:95,108)."""
    return torch.linspace(-.2, .2, n, dtype=dtype, device=device)


def poisoned_view(x: torch.Tensor, layout: str, device: str | torch.device) -> torch.Tensor:
    """Rebuild ``x`` on ``device`` inside NaN-filled storage.

    layouts: ``padded`` (row stride cols + 8), ``transposed`` (column-major
    storage, so the view has strides (1, rows)), ``offset`` (base shifted by
    one element: not 16-byte aligned), ``strided`` (every other element,
    qualification.py:66-72).
    """
    rows, cols = x.shape
    if layout == "padded":
        store = torch.full((rows, cols + 8), float("nan"), dtype=x.dtype, device=device)
        store[:, :cols] = x.to(device)
        return store[:, :cols]
    if layout == "transposed":
        store = torch.full((cols, rows), float("nan"), dtype=x.dtype, device=device)
        store.copy_(x.t().to(device))
        return store.t()
    if layout == "offset":
        store = torch.full((rows * cols + 16,), float("nan"), dtype=x.dtype, device=device)
        view = store[1:1 + rows * cols].view(rows, cols)
        view.copy_(x.to(device))
        return view
    if layout == "strided":
        store = torch.full((rows, cols * 2 + 2), float("nan"), dtype=x.dtype, device=device)
        store[:, 1:1 + 2 * cols:2] = x.to(device)
        return store[:, 1:1 + 2 * cols:2]
    raise ValueError(layout)


def sha256_of(*tensors: torch.Tensor) -> str:
    """sha256 over the raw little-endian bytes of contiguous copies."""
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()
