"""Timing and statistics of the qualification harness.

* ``stats``          -- p05/p50/p95/MAD summary (evidence.py:63-69 of the
  reference), same keys.
* ``torch_measure``  -- the reference's randomised-order CUDA-event loop
  (evidence.py:87-105): per round a fresh shuffle of the functions, each
  timed over ``inner`` back-to-back calls.  With two functions this is the
  randomised AB/BA pair protocol.
* ``device_measure`` -- the same event protocol without host dispatch gaps:
  each sample first enqueues a short GPU hold (``torch.cuda._sleep``) so the
  ``inner`` launches behind it are all queued before the GPU reaches them;
  the event pair then spans exactly ``inner`` back-to-back calls of device
  work.  ``inner = 1`` gives the isolated single-call latency, which also
  contains the device-side launch latency of that one kernel.
"""
from __future__ import annotations

import math
import random
import statistics
from typing import Callable


def stats(values: list[float]) -> dict:
    if not values or any(not math.isfinite(v) or v < 0 for v in values):
        raise ValueError("expected nonempty finite nonnegative measurements")
    s = sorted(values)
    med = statistics.median(s)
    return {"n": len(s), "p50_ms": med, "p05_ms": s[int(.05 * (len(s) - 1))],
            "p95_ms": s[int(.95 * (len(s) - 1))], "mean_ms": statistics.fmean(s),
            "mad_ms": statistics.median(abs(v - med) for v in s)}


def torch_measure(functions: dict[str, Callable[[], object]], samples: int = 31, warmup: int = 20,
                  inner: int = 10, seed: int = 1729) -> dict:
    """The reference's protocol; warmup defaults to 20 calls, as the headline metric specifies."""
    import torch
    if samples < 3 or warmup < 0 or inner < 1:
        raise ValueError("invalid benchmark parameters")
    for f in functions.values():
        for _ in range(warmup):
            f()
    torch.cuda.synchronize()
    rng = random.Random(seed)
    raw = {k: [] for k in functions}
    order = []
    for _ in range(samples):
        keys = list(functions)
        rng.shuffle(keys)
        order.append(keys)
        for key in keys:
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            start.record()
            for _ in range(inner):
                functions[key]()
            end.record()
            end.synchronize()
            raw[key].append(start.elapsed_time(end) / inner)
    return {"order": order, "inner": inner, "warmup": warmup, "seed": seed,
            "measurements": {k: {"cuda_event": stats(v), "raw_ms": v} for k, v in raw.items()}}


def hold_cycles(microseconds: float) -> int:
    """Cycles for torch.cuda._sleep at the B200's 1.965 GHz boost clock."""
    return int(microseconds * 1965)


def device_measure(functions: dict[str, Callable[[], object]], rounds: int, inner: int = 10, seed: int = 7,
                   hold_us: float = 400.0, align: Callable[[], object] | None = None) -> dict[str, list[float]]:
    """Per-call device milliseconds, ``rounds`` samples per function.

    Each sample: a GPU hold of ``hold_us`` (so the launches behind it queue
    up), a start event, ``inner`` back-to-back calls, an end event, all on the
    current stream; the sample is the span / ``inner``.  Functions are visited
    in a fresh shuffled order every round.  Returns the raw samples.

    ``align`` (multi-GPU): enqueued before each sample's hold, it lines the
    ranks' streams up on the device (e.g. a one-element collective), so that
    every rank's hold ends at the same moment and a call that waits for its
    peers does not absorb the ranks' host launch skew.
    """
    import torch
    stream = torch.cuda.current_stream()
    rng = random.Random(seed)
    raw = {k: [] for k in functions}
    keys = list(functions)
    events = {k: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for k in keys}
    for _ in range(rounds):
        rng.shuffle(keys)
        for key in keys:
            start, end = events[key]
            if align is not None:
                align()
            torch.cuda._sleep(hold_cycles(hold_us))
            start.record(stream)
            fn = functions[key]
            for _ in range(inner):
                fn()
            end.record(stream)
        stream.synchronize()
        for key in keys:
            start, end = events[key]
            raw[key].append(start.elapsed_time(end) / inner)
    return raw
