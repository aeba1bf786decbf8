#!/usr/bin/env python
"""Benchmark of the FP16 linear + bias + SiLU fragment on B200.

Workload (the headline configs, N = K = 4096): y = SiLU(A @ W^T + b) and y = A @ W^T with
A [M, 4096], W [4096, 4096] (K-contiguous), b [4096], seed-7 uniform
[-0.5, 0.5) FP16 inputs, for M in {1, 8, 32, 128}.  One *step* runs the eight
calls (four M values x {fused, plain}) in a freshly shuffled order, each call
on its own rotating copy of W so that every call streams W from HBM (the
copies together exceed the L2).  The headline ``value`` is the p50 device
latency of the fused M = 32 call; ``sweep`` holds every M.

Timing (the reference's evidence.torch_measure protocol, inner = 10): a
sample is one event pair on the launching stream around 10 back-to-back calls
of one variant, each call on the next rotating W copy, queued behind a short
GPU hold so host dispatch never shows in the span; per-call time = span / 10.
The isolated single-call latency (inner = 1, includes the device-side launch
latency of one kernel) is reported next to it in ``sweep``.

Also reported: the roofline of the dominant kernel against the measured HBM
peak (MEASURED_PEAKS.json), warm-L2 numbers (one W copy), an end-to-end number
through the public operator API with pinned host buffers and the copies inside
the timed region, the CPU FP64 oracle timed on the host cores, and SM clocks
sampled during the timed region.

Multi-GPU (torchrun, one rank per GPU): column-parallel sharding of the same
fused M = 32 layer, W split along N into equal slices, local fused GEMM, NCCL
all-gather of the [M, N/P] outputs and the [P, M, N/P] -> [M, N] layout fix;
device-timed, max over ranks.

``--impl reference``: the reference's CPU implementation of the path (the FP64
oracle port of qualification.reference) on the host cores, same metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "p50 latency (μs) and % HBM roofline, FP16 GEMM+bias+SiLU, M=1..128, N=K=4096"
N_DIM = K_DIM = 4096
SWEEP_M = (1, 8, 32, 128)
FALLBACK_HBM_GBS = 6650.0
DATA = ("synthetic: seed-7 uniform [-0.5, 0.5) FP32 draws (torch.Generator, order A, W, bias) rounded to "
        "FP16; W [N, K] row-major")


def algorithmic_bytes(m: int, n: int = N_DIM, k: int = K_DIM, bias: bool = True) -> int:
    """2 * (M*K + N*K + M*N) (+ 2*N for the bias): each operand once."""
    return 2 * (m * k + n * k + m * n) + (2 * n if bias else 0)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["native", "reference"], default="native")
    p.add_argument("--m", type=int, default=32, help="M of the headline value")
    p.add_argument("--copies", type=int, default=0, help="rotating W copies (0 = from the L2 size)")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-probes", action="store_true", help="skip the boundary and split-K probe timings")
    p.add_argument("--inner", type=int, default=10, help="back-to-back calls per timed sample")
    p.add_argument("--sweep", type=str, default=",".join(map(str, SWEEP_M)),
                   help="comma-separated M values of the step (default 1,8,32,128)")
    p.add_argument("--no-sharded-shapes", action="store_true",
                   help="N > 1: skip the column-parallel shapes (N = 8192 / 28672, K = 8192)")
    return p.parse_args(argv)


# ---------------------------------------------------------------- helpers

def measured_hbm_peak() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        peaks = json.loads(path.read_text())
        return float(peaks["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def profiled_traffic(kernel_tag: str) -> int | None:
    """DRAM bytes per launch recorded by an ncu capture summary in profiles/.

    The summary files carry a line ``dram_bytes_per_launch[<tag>]: <int>``.
    """
    for path in sorted((REPO / "profiles").glob("*.md")):
        for line in path.read_text().splitlines():
            key = f"dram_bytes_per_launch[{kernel_tag}]:"
            if line.strip().startswith(key):
                try:
                    return int(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """SM clocks, power and clock-event reasons sampled DURING a timed region.

    NVML (read-only queries) is polled from a thread every 10 ms, with one
    sample taken on entry, so that even a region of a few milliseconds is
    covered; without NVML, ``nvidia-smi -lms 100`` is the fallback.  The NVML
    device is found by the CUDA device's UUID, so CUDA_VISIBLE_DEVICES
    renumbering does not pick another GPU.
    """

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.01
    # NVML clock-event reason bits (nvml.h nvmlClocksEventReason*).
    REASON_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                   ("sw_power_cap", 0x4))

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None
        self.nvml = None
        self.handle = None
        self.rows: list[dict] = []
        self.stop = None
        self.thread = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        self.nvml = pynvml
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _nvml_sample(self) -> None:
        nv, h = self.nvml, self.handle
        reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        self.rows.append({"sm": float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                          "max": float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)),
                          "power": nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                          "reasons": [name for name, bit in self.REASON_BITS if reasons & bit]})

    def _poll(self) -> None:
        while not self.stop.wait(self.PERIOD_S):
            try:
                self._nvml_sample()
            except Exception:
                return

    def __enter__(self):
        try:
            self.handle = self._nvml_handle()
            self._nvml_sample()
            import threading
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.handle = None
            self.rows = []
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def _smi_rows(self) -> list[dict]:
        if self.proc is None or self.file is None:
            return []
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                flags = dict(zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 parts[5:9]))
                rows.append({"sm": float(parts[1]), "max": float(parts[2]), "power": float(parts[3]),
                             "reasons": [k for k, v in flags.items() if v.lower() == "active"]})
            except ValueError:
                continue
        os.unlink(self.file.name)
        return rows

    def summary(self) -> dict | None:
        rows = self.rows if self.handle is not None else self._smi_rows()
        if not rows:
            return None
        reasons = sorted({r for row in rows for r in row["reasons"]})
        return {"sm_mhz": statistics.median(r["sm"] for r in rows), "sm_max_mhz": max(r["max"] for r in rows),
                "power_w_max": max(r["power"] for r in rows), "samples": len(rows), "reasons": reasons,
                "source": "nvml" if self.handle is not None else "nvidia-smi"}


def host_threads() -> int:
    """Cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def use_all_host_threads() -> None:
    """Let the BLAS behind numpy use every core (torchrun sets OMP_NUM_THREADS=1)."""
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=host_threads(), user_api="blas")
    except Exception:  # threadpoolctl missing: keep the library default
        pass


def numpy_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        return max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:  # threadpoolctl missing: report the core count numpy may use
        return os.cpu_count() or 1


# ---------------------------------------------------------------- CPU legs

def cpu_fragment_timings(m: int, budget_s: float, max_calls: int) -> tuple[list[float], dict]:
    """FP64 SiLU(A @ W^T + b) on the host cores: the oracle's compute core."""
    import numpy as np
    use_all_host_threads()
    from gemm_lab_qualification_b200 import workloads
    from oracle import reference as oracle
    a, w, bias = workloads.uniform_inputs(m, N_DIM, K_DIM)
    a64 = a.double().numpy()
    wt64 = np.ascontiguousarray(w.double().numpy().T)
    b64 = bias.double().numpy()
    oracle.silu_reference(a64 @ wt64, b64)  # warm-up (BLAS threads, pages)
    times = []
    start = time.perf_counter()
    while len(times) < max_calls and (time.perf_counter() - start < budget_s or len(times) < 3):
        t0 = time.perf_counter()
        oracle.silu_reference(a64 @ wt64, b64)
        times.append((time.perf_counter() - t0) * 1e6)
    t0 = time.perf_counter()
    oracle.linear_reference(a, w, bias, silu=True)  # with the 64-dot fsum cross-check
    full_us = (time.perf_counter() - t0) * 1e6
    info = {"cores": numpy_threads(), "reference_full_call_us": full_us,
            "sample": f"{len(times)} calls of the full M={m} fused fragment (N=K=4096) in FP64 numpy; "
                      f"reference_full_call_us adds the 64-dot math.fsum cross-check of qualification.reference"}
    return times, info


def run_reference_arm(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    budget = max(5.0, args.cpu_seconds)
    for _ in range(min(args.warmup, 3)):
        cpu_fragment_timings(args.m, 0.0, 1)
    times, info = cpu_fragment_timings(args.m, budget, max(args.steps, 3))
    p50 = statistics.median(times)
    line = {"metric": METRIC, "value": p50, "unit": "us", "n_gpus": args.gpus, "steps": len(times),
            "warmup": args.warmup, "ms_per_step": statistics.fmean(times) / 1e3, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": DATA,
            "config": {"workload": f"fused linear+bias+SiLU, M={args.m}, N=K=4096 (CPU FP64 oracle port)",
                       "m": args.m, "n": N_DIM, "k": K_DIM, "parallelism": "host cores"},
            "impl": "reference",
            "cpu_baseline": {"value": p50, "unit": "us", "cores": info["cores"], "kind": "port",
                             "sample": info["sample"], "reference_full_call_us": info["reference_full_call_us"]},
            "e2e": {"value": p50, "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU legs

def single_gpu(args, torch, dev) -> dict:
    from gemm_lab_qualification_b200 import kernels, workloads
    from gemm_lab_qualification_b200.evidence import device_measure

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    props = torch.cuda.get_device_properties(dev)
    l2 = int(getattr(props, "L2_cache_size", 126 * 2 ** 20))
    w_bytes = N_DIM * K_DIM * 2
    copies = args.copies or max(4, math.ceil(3 * l2 / w_bytes))
    sweep_m = sorted({int(x) for x in args.sweep.split(",") if x} | {args.m})

    state = {}
    for m in sweep_m:
        a, w, bias = workloads.uniform_inputs(m, N_DIM, K_DIM)
        da, db = a.to(dev), bias.to(dev)
        ws = [w.to(dev) for _ in range(copies)]
        # The lab harness's own operand layout, B = [K, N] row-major.
        ws_kn = [w.t().contiguous().to(dev) for _ in range(copies)]
        state[m] = {"a": da, "w": ws, "w_kn": ws_kn, "bias": db, "fused": torch.empty((m, N_DIM), dtype=torch.float16, device=dev),
                    "plain": torch.empty((m, N_DIM), dtype=torch.float16, device=dev), "i": 0}

    # Gate before timing (the harness refuses to time wrong output): torch
    # FP32 reference on the device, TF32 off, the uniform-corpus tolerance.
    paths = {}
    for m, st in state.items():
        kernels.triton_bias_silu_into(st["a"], st["w"][0].t(), st["bias"], st["fused"])
        paths[m] = kernels.last_path()
        ref = torch.nn.functional.silu(st["a"].float() @ st["w"][0].float().t() + st["bias"].float())
        err = (st["fused"].float() - ref).abs()
        if not bool((err <= 0.02 + 0.002 * ref.abs()).all()):
            raise SystemExit(f"correctness gate failed at M={m}: max abs error {float(err.max())}")
        kernels.triton_matmul_into(st["a"], st["w"][0].t(), st["plain"])
        ref = st["a"].float() @ st["w"][0].float().t()
        err = (st["plain"].float() - ref).abs()
        if not bool((err <= 0.02 + 0.002 * ref.abs()).all()):
            raise SystemExit(f"correctness gate failed (plain) at M={m}")
        kernels.triton_bias_silu_into(st["a"], st["w_kn"][0], st["bias"], st["fused"])
        paths[f"kn{m}"] = kernels.last_path()
        ref = torch.nn.functional.silu(st["a"].float() @ st["w_kn"][0].float() + st["bias"].float())
        err = (st["fused"].float() - ref).abs()
        if not bool((err <= 0.02 + 0.002 * ref.abs()).all()):
            raise SystemExit(f"correctness gate failed (B = [K, N]) at M={m}")
    torch.cuda.synchronize()

    def call(m, variant, rotate=True):
        st = state[m]

        def run():
            w = st["w"][st["i"] % copies] if rotate else st["w"][0]
            st["i"] += 1
            if variant == "fused":
                kernels.triton_bias_silu_into(st["a"], w.t(), st["bias"], st["fused"])
            else:
                kernels.triton_matmul_into(st["a"], w.t(), st["plain"])
        return run

    fns = {f"{v}/m{m}": call(m, v) for m in sweep_m for v in ("fused", "plain")}
    device_measure(fns, rounds=args.warmup, inner=args.inner)
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks:
        t0 = time.perf_counter()
        raw = device_measure(fns, rounds=args.steps, inner=args.inner)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    isolated = device_measure(fns, rounds=max(10, args.steps // 4), inner=1)
    # Same-round vendor comparator, same protocol and rotating W copies:
    # cuBLASLt through torch (F.linear = GEMM with the bias epilogue, then a
    # separate SiLU kernel: equal semantics except that the bias epilogue
    # rounds to FP16 before the SiLU) and the plain GEMM (torch.mm).
    def vendor(m, variant):
        st = state[m]

        def run():
            w = st["w"][st["i"] % copies]
            st["i"] += 1
            if variant == "fused":
                torch.nn.functional.silu(torch.nn.functional.linear(st["a"], w, st["bias"]), inplace=True)
            else:
                torch.mm(st["a"], w.t(), out=st["plain"])
        return run

    cublas = device_measure({f"{v}/m{m}": vendor(m, v) for m in sweep_m for v in ("fused", "plain")},
                            rounds=max(10, args.steps // 3), inner=args.inner)

    # The lab harness's own protocol (evidence.torch_measure: no GPU hold, so
    # host dispatch is inside the span; the same resident W every call, warm
    # L2; 20 warm-ups, 31 randomised samples of 10 calls): what
    # qualification.benchmark() would report for the drop-in operators.
    from gemm_lab_qualification_b200.evidence import torch_measure
    lab = {}
    for m in sweep_m:
        st = state[m]
        w0 = st["w"][0]
        res = torch_measure({
            "ours": lambda st=st, w0=w0: kernels.triton_bias_silu_into(st["a"], w0.t(), st["bias"], st["fused"]),
            "torch": lambda st=st, w0=w0: torch.nn.functional.silu(
                torch.nn.functional.linear(st["a"], w0, st["bias"]), inplace=True),
        }, samples=31, warmup=20, inner=args.inner)
        lab[m] = {k: v["cuda_event"]["p50_ms"] * 1e3 for k, v in res["measurements"].items()}

    # The fused call on the lab's own B = [K, N] operand (MN-major W tiles).
    def b_kn(m):
        st = state[m]

        def run():
            w_kn = st["w_kn"][st["i"] % copies]
            st["i"] += 1
            kernels.triton_bias_silu_into(st["a"], w_kn, st["bias"], st["fused"])
        return run

    kn = device_measure({f"fused/m{m}": b_kn(m) for m in sweep_m}, rounds=max(10, args.steps // 3),
                        inner=args.inner)
    # Launch modes of the fused calls: without programmatic dependent launch,
    # and with the inference declaration that W is static.
    modes = {}
    fused_fns = {k: f for k, f in fns.items() if k.startswith("fused/")}
    for label, opts in (("no_pdl", {"pdl": False}), ("static_weights", {"static_weights": True})):
        with kernels.launch_options(**opts):
            modes[label] = device_measure(fused_fns, rounds=max(10, args.steps // 3), inner=args.inner)
    # Warm L2: one variant at a time on a single W copy (32 MiB fits in L2).
    warm = {}
    for key in fns:
        m_key, v_key = int(key.split("/m")[1]), key.split("/")[0]
        warm.update(device_measure({key: call(m_key, v_key, rotate=False)}, rounds=max(5, args.steps // 10),
                                   inner=args.inner))

    # The MLP shapes gated by the lab's adaptive_bias_silu_path (4096 <-> 11008,
    # kernels.py:295): fused call vs the cuBLASLt fragment, rotating weights.
    mlp = []
    for n_m, k_m in ((11008, 4096), (4096, 11008)):
        w_bytes_m = n_m * k_m * 2
        copies_m = max(4, math.ceil(3 * l2 / w_bytes_m))
        for m in (1, 32):
            a_m, w_m, b_m = workloads.uniform_inputs(m, n_m, k_m)
            da_m, db_m = a_m.to(dev), b_m.to(dev)
            ws_m = [w_m.to(dev) for _ in range(copies_m)]
            y_m = torch.empty((m, n_m), dtype=torch.float16, device=dev)
            cnt = {"i": 0}

            def ours(da_m=da_m, db_m=db_m, ws_m=ws_m, y_m=y_m, cnt=cnt, copies_m=copies_m):
                cnt["i"] += 1
                kernels.triton_bias_silu_into(da_m, ws_m[cnt["i"] % copies_m].t(), db_m, y_m)

            def theirs(da_m=da_m, db_m=db_m, ws_m=ws_m, cnt=cnt, copies_m=copies_m):
                cnt["i"] += 1
                torch.nn.functional.silu(torch.nn.functional.linear(da_m, ws_m[cnt["i"] % copies_m], db_m),
                                         inplace=True)
            ours()
            path_m = kernels.last_path()
            fns_m = {"ours": ours, "cublas": theirs}
            device_measure(fns_m, rounds=3, inner=args.inner)
            raw_m = device_measure(fns_m, rounds=max(10, args.steps // 5), inner=args.inner)
            us = statistics.median(raw_m["ours"]) * 1e3
            mlp.append({"m": m, "n": n_m, "k": k_m, "path": list(path_m), "fused_p50_us": us,
                        "cublas_fused_p50_us": statistics.median(raw_m["cublas"]) * 1e3,
                        "gbs": 2 * (m * k_m + n_m * k_m + m * n_m + n_m) / (us * 1e-6) / 1e9})
            del ws_m
    peak, peak_src = measured_hbm_peak()
    sweep = {}
    for m in sweep_m:
        row = {"path": paths[m][0], "split": paths[m][1], "bytes_fused": algorithmic_bytes(m),
               "bytes_plain": algorithmic_bytes(m, bias=False)}
        for v in ("fused", "plain"):
            samples = raw[f"{v}/m{m}"]
            p50_ms = statistics.median(samples)
            mean_ms = statistics.fmean(samples)
            gbs = row[f"bytes_{v}"] / (p50_ms * 1e-3) / 1e9
            row[f"{v}_p50_us"] = p50_ms * 1e3
            row[f"{v}_mean_us"] = mean_ms * 1e3
            row[f"{v}_p05_us"] = sorted(samples)[int(.05 * (len(samples) - 1))] * 1e3
            row[f"{v}_p95_us"] = sorted(samples)[int(.95 * (len(samples) - 1))] * 1e3
            row[f"{v}_gbs"] = gbs
            row[f"{v}_frac"] = gbs / peak
            row[f"{v}_warm_l2_p50_us"] = statistics.median(warm[f"{v}/m{m}"]) * 1e3
            row[f"{v}_isolated_p50_us"] = statistics.median(isolated[f"{v}/m{m}"]) * 1e3
        for label, samples in modes.items():
            row[f"fused_{label}_p50_us"] = statistics.median(samples[f"fused/m{m}"]) * 1e3
        for v in ("fused", "plain"):
            row[f"cublas_{v}_p50_us"] = statistics.median(cublas[f"{v}/m{m}"]) * 1e3
        row["fused_b_kn_p50_us"] = statistics.median(kn[f"fused/m{m}"]) * 1e3
        row["fused_lab_protocol_p50_us"] = lab[m]["ours"]
        row["torch_fragment_lab_protocol_p50_us"] = lab[m]["torch"]
        row["b_kn_path"] = paths[f"kn{m}"][0]
        sweep[str(m)] = row

    head = sweep[str(args.m)]
    mean_s = head["fused_mean_us"] * 1e-6
    achieved = head["bytes_fused"] / mean_s / 1e9
    # profiles/*.md record DRAM bytes per launch under "<kernel>_m<M>" tags
    kernel_tag = "gemv" if head["path"] == "gemv_m1" else "tc_linear"
    traffic = profiled_traffic(f"{kernel_tag}_m{args.m}")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "peak_source": peak_src,
                "kernel": f"{kernel_tag} (fused, M={args.m}, path {head['path']}, split {head['split']})",
                "algorithmic_bytes_per_launch": head["bytes_fused"], "launch_mean_us": head["fused_mean_us"]}
    ms_per_step = sum(statistics.fmean(v) for v in raw.values()) * args.inner
    return {"value": head["fused_p50_us"], "ms_per_step": ms_per_step, "sweep": sweep, "mlp_shapes": mlp,
            "roofline": roofline,
            "clocks": clocks.summary(), "copies": copies, "l2_bytes": l2, "wall_s": wall,
            "gpu_launches": args.steps * len(fns) * args.inner, "state": state}


PROBE_A_VIEWS = {"a_padded": "padded", "a_transposed": "transposed", "a_offset": "offset"}


def probe_timings(args, torch, dev) -> dict:
    """The manifest's boundary probes and the forced split-K probes, timed.

    Each probe runs through the operator API (triton_bias_silu_into, or
    triton_splitk_matmul_into with a caller FP32 [S, M, N] partial buffer) and
    is timed like the sweep: p50 of `inner` back-to-back calls behind a GPU
    hold, the weight rotating over copies larger than L2.  GB/s counts the
    algorithmic bytes; the split partials' write-back is inside the timed
    region but not counted.
    """
    from gemm_lab_qualification_b200 import kernels, workloads
    from gemm_lab_qualification_b200.evidence import device_measure
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    peak, _ = measured_hbm_peak()
    rounds = max(10, args.steps // 10)

    def copies_for(nbytes: int) -> int:
        return max(2, -(-2 * l2 // nbytes) + 1) if nbytes else 1

    def measure(fn) -> float:
        fn()
        device_measure({"p": fn}, rounds=2, inner=args.inner)
        return statistics.median(device_measure({"p": fn}, rounds=rounds, inner=args.inner)["p"]) * 1e3

    boundary = []
    for probe in workloads.MANIFEST["probes"]:
        m, n, k, layout = probe["m"], probe["n"], probe["k"], probe["layout"]
        a, w, bias = workloads.uniform_inputs(m, n, k)
        da = workloads.poisoned_view(a, PROBE_A_VIEWS[layout], dev) if layout in PROBE_A_VIEWS else a.to(dev)
        copies = copies_for(w.numel() * 2)
        wts = [workloads.poisoned_view(w, "padded", dev) if layout == "w_padded" else w.to(dev)
               for _ in range(copies)]
        db = bias.to(dev)
        y = torch.empty((m, n), dtype=torch.float16, device=dev)
        cnt = {"i": 0}

        def call(da=da, wts=wts, db=db, y=y, cnt=cnt):
            cnt["i"] += 1
            kernels.triton_bias_silu_into(da, wts[cnt["i"] % len(wts)].t(), db, y)
        us = measure(call)
        path = kernels.last_path()
        nbytes = algorithmic_bytes(m, n, k) if m and n else 0
        gbs = nbytes / (us * 1e-6) / 1e9 if nbytes and us > 0 else None
        boundary.append({"id": probe["id"], "m": m, "n": n, "k": k, "layout": layout, "path": path[0],
                         "split": path[1], "p50_us": us, "gbs": gbs, "frac": gbs / peak if gbs else None})
        del wts
    split = []
    sp = workloads.MANIFEST["split_probes"]
    _, w, _ = workloads.uniform_inputs(1, sp["n"], sp["k"])
    wts = [w.to(dev) for _ in range(copies_for(w.numel() * 2))]
    for m in sp["m"]:
        a, _, _ = workloads.uniform_inputs(m, sp["n"], sp["k"])
        da = a.to(dev)
        y = torch.empty((m, sp["n"]), dtype=torch.float16, device=dev)
        for s in sp["splits"]:
            partial = torch.empty((s, m, sp["n"]), dtype=torch.float32, device=dev)
            cnt = {"i": 0}

            def call(da=da, partial=partial, y=y, s=s, cnt=cnt):
                cnt["i"] += 1
                kernels.triton_splitk_matmul_into(da, wts[cnt["i"] % len(wts)].t(), partial, y, s)
            us = measure(call)
            path = kernels.last_path()
            gbs = algorithmic_bytes(m, sp["n"], sp["k"], bias=False) / (us * 1e-6) / 1e9
            split.append({"m": m, "split": s, "path": path[0], "reported_split": path[1], "p50_us": us,
                          "gbs": gbs, "frac": gbs / peak, "partial_bytes": s * m * sp["n"] * 4})
    del wts
    return {"protocol": f"operator API, p50 of {args.inner} back-to-back calls behind a GPU hold, {rounds} "
                        "samples, weight rotating over copies > L2", "boundary": boundary, "split": split}


def e2e_public_api(args, torch, dev, rounds: int) -> dict:
    """Host buffers in, host result out, through kernels.triton_bias_silu_into.

    The host-to-host pipeline of qualification.py:114-117: each step copies
    the call's inputs from pinned host memory to the device, runs the
    operator and copies Y back.  The inputs sit in ONE pinned staging buffer
    (W, then A, then the bias, each 256-byte aligned) mirrored by one device
    buffer, so a step is one H2D copy, one kernel and one D2H copy; with
    resident weights only the A + bias part is copied.
    """
    from gemm_lab_qualification_b200 import kernels, workloads
    m = args.m
    a, w, bias = workloads.uniform_inputs(m, N_DIM, K_DIM)

    def align(nbytes: int) -> int:
        return (nbytes + 255) // 256 * 256

    w_bytes, a_bytes, b_bytes = w.numel() * 2, a.numel() * 2, bias.numel() * 2
    offs = {"w": 0, "a": align(w_bytes), "bias": align(w_bytes) + align(a_bytes)}
    total = offs["bias"] + align(b_bytes)
    h_in = torch.empty(total, dtype=torch.uint8).pin_memory()
    d_in = torch.empty(total, dtype=torch.uint8, device=dev)

    def view(buf, key, t):
        n = t.numel() * 2
        return buf[offs[key]:offs[key] + n].view(torch.float16).view(t.shape)

    view(h_in, "w", w).copy_(w)
    view(h_in, "a", a).copy_(a)
    view(h_in, "bias", bias).copy_(bias)
    dw, da, db = view(d_in, "w", w), view(d_in, "a", a), view(d_in, "bias", bias)
    hy = torch.empty((m, N_DIM), dtype=torch.float16).pin_memory()
    dy = torch.empty((m, N_DIM), dtype=torch.float16, device=dev)

    def step(copy_weights: bool):
        lo = 0 if copy_weights else offs["a"]
        d_in[lo:].copy_(h_in[lo:], non_blocking=True)
        kernels.triton_bias_silu_into(da, dw.t(), db, dy)
        hy.copy_(dy, non_blocking=True)

    d_in.copy_(h_in)
    out = {}
    for label, copy_weights in (("all_inputs", True), ("resident_weights", False)):
        for _ in range(3):
            step(copy_weights)
        torch.cuda.synchronize()
        samples, walls = [], []
        for _ in range(rounds):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            start.record()
            step(copy_weights)
            end.record()
            end.synchronize()
            walls.append((time.perf_counter() - t0) * 1e6)
            samples.append(start.elapsed_time(end) * 1e3)
            _ = float(hy[0, 0])  # the host consumes the result
        h2d = total - (0 if copy_weights else offs["a"])
        out[label] = {"value": statistics.median(samples), "unit": "us", "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": hy.numel() * 2, "wall_p50_us": statistics.median(walls),
                      "copies_per_step": {"h2d": 1, "d2h": 1}}
    if not torch.equal(dy.cpu(), hy):
        raise SystemExit("e2e: the host copy of Y differs from the device result")
    return out


def multi_gpu(args, torch, dist, dev, world: int, rank: int) -> dict:
    """Column-parallel fused layer on `world` GPUs, weak scaling: every rank
    owns a 4096-row slice of W (the single-GPU fragment's weight), so
    N = 4096 * world, K = 4096, M = args.m.  Headline: the fused-gather layer
    (one kernel per rank: tcgen05 GEMM whose epilogue stores into every
    rank's output over NVLink, then an epoch handshake).  Comparator: the same
    local kernel followed by an NCCL all-gather and the layout copy."""
    from gemm_lab_qualification_b200 import _native, kernels, sharded, workloads
    from gemm_lab_qualification_b200.evidence import device_measure
    m = args.m
    n_total = N_DIM * world
    a, w, bias = workloads.uniform_inputs(m, n_total, K_DIM)
    layer = sharded.ColumnParallelLinear(w, bias, "silu", device=dev, fused_gather=True, max_rows=m)
    ns = layer.weight.shape[0]
    props = torch.cuda.get_device_properties(dev)
    l2 = int(getattr(props, "L2_cache_size", 126 * 2 ** 20))
    copies = args.copies or max(4, math.ceil(3 * l2 / (ns * K_DIM * 2)))
    ws = [layer.weight.clone() for _ in range(copies)]
    da = a.to(dev)
    local = torch.empty((m, ns), dtype=torch.float16, device=dev)
    gathered = torch.empty((world, m, ns), dtype=torch.float16, device=dev)
    y_nccl = torch.empty((m, n_total), dtype=torch.float16, device=dev)
    state = {"i": 0}
    epi = _native.EPILOGUE_BIAS_SILU

    def fused_step():
        wi = ws[state["i"] % copies]
        state["i"] += 1
        return layer.gather(da, wi.t(), layer.bias, epi)

    def nccl_step():
        wi = ws[state["i"] % copies]
        state["i"] += 1
        kernels.triton_bias_silu_into(da, wi.t(), layer.bias, local)
        sharded.gather_columns(local, y_nccl, gathered=gathered)

    # Correctness gate on every rank (torch FP32 reference, the uniform-corpus tolerance).
    y_fused = fused_step().clone()
    nccl_step()
    torch.cuda.synchronize()
    wd = w.to(dev)
    ref = torch.nn.functional.silu(da.float() @ wd.float().t() + bias.to(dev).float())
    del wd
    for label, y in (("fused", y_fused), ("nccl", y_nccl)):
        err = (y.float() - ref).abs()
        if not bool((err <= 0.02 + 0.002 * ref.abs()).all()):
            raise SystemExit(f"rank {rank}: sharded correctness gate failed ({label})")
    path = kernels.last_path()
    if _native.device_error(clear=True):
        raise SystemExit(f"rank {rank}: a bounded in-kernel wait expired")
    # Each function is timed alone, identically on every rank (the fused
    # kernels of one call wait for each other across GPUs).
    # The GPU hold must outlast the host's enqueueing of `inner` calls (the
    # NCCL comparator's Python + collective launch costs dominate there).
    host_us = {}
    for label, fn in (("fused", fused_step), ("nccl", nccl_step)):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.inner):
            fn()
        host_us[label] = (time.perf_counter() - t0) * 1e6 / args.inner
        torch.cuda.synchronize()
    hold = max(400.0, 3.0 * args.inner * max(host_us.values()))
    # Every sample starts with the ranks' streams lined up on the device (a
    # one-element all-reduce), so the timed calls measure the layer in step,
    # as consecutive layers of a model run, not the ranks' host launch skew.
    token = torch.zeros(1, dtype=torch.float32, device=dev)
    align = lambda: dist.all_reduce(token)
    raws = {}
    for label, fn in (("fused", fused_step), ("nccl", nccl_step)):
        device_measure({label: fn}, rounds=args.warmup, inner=args.inner, hold_us=hold, align=align)
        dist.barrier()
        torch.cuda.synchronize()
        with ClockSampler(dev.index) as clocks:
            raws[label] = device_measure({label: fn}, rounds=args.steps, inner=args.inner, hold_us=hold,
                                         align=align)[label]
            torch.cuda.synchronize()
        if label == "fused":
            clock_summary = clocks.summary()
        dist.barrier()
    if _native.device_error(clear=True):
        raise SystemExit(f"rank {rank}: a bounded in-kernel wait expired while timing")

    # End to end through the public layer API: pinned host A, this rank's W
    # slice and bias in, the gathered Y out, every step.
    ha = a.pin_memory()
    hw = layer.weight.cpu().pin_memory()
    hb = layer.bias.cpu().pin_memory()
    hy = torch.empty((m, n_total), dtype=torch.float16).pin_memory()
    dw = torch.empty_like(layer.weight)
    db = torch.empty_like(layer.bias)

    def e2e_step():
        da.copy_(ha, non_blocking=True)
        dw.copy_(hw, non_blocking=True)
        db.copy_(hb, non_blocking=True)
        y = layer.gather(da, dw.t(), db, epi)
        hy.copy_(y, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    e2e = []
    for _ in range(max(10, args.steps // 4)):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        e2e_step()
        end.record()
        end.synchronize()
        _ = float(hy[0, 0])
        e2e.append(start.elapsed_time(end) * 1e3)
    dist.barrier()
    stats = torch.tensor([statistics.median(raws["fused"]), statistics.fmean(raws["fused"]),
                          statistics.median(raws["nccl"]), statistics.median(e2e)], dtype=torch.float64, device=dev)
    dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    return {"value": float(stats[0]) * 1e3, "mean_us": float(stats[1]) * 1e3, "nccl_us": float(stats[2]) * 1e3,
            "e2e_us": float(stats[3]), "path": path, "clocks": clock_summary, "shard_rows": ns, "n_total": n_total,
            "copies": copies, "gpu_launches": args.steps * args.inner * 2, "host_us": host_us, "hold_us": hold,
            "h2d": ha.numel() * 2 + hw.numel() * 2 + hb.numel() * 2, "d2h": hy.numel() * 2}


SHARDED_SHAPES = ((8192, 8192), (28672, 8192))  # (N, K) of the column-parallel configs
SHARDED_M = (1, 32, 128, 4096)


def sharded_shapes(args, torch, dist, dev, world: int, rank: int) -> list[dict]:
    """The column-parallel shapes, strong scaling: W [N, K] split along N
    over the ranks, fused bias+SiLU, all-gather fused into the kernel.  Inputs
    are uniform [-0.5, 0.5) draws of the device generator seeded 7 (the full
    layer is generated identically on every rank and sliced).  Rank 0 also
    times the unsharded layer alone on its GPU for the same shape."""
    from gemm_lab_qualification_b200 import _native, sharded
    from gemm_lab_qualification_b200.evidence import device_measure
    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    tensor_peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
    out = []
    for n_total, k in SHARDED_SHAPES:
        gen = torch.Generator(device=dev).manual_seed(7)
        w = (torch.rand((n_total, k), generator=gen, device=dev, dtype=torch.float32) - 0.5).half()
        bias = (torch.rand((n_total,), generator=gen, device=dev, dtype=torch.float32) - 0.5).half()
        for m in SHARDED_M:
            a = (torch.rand((m, k), generator=gen, device=dev, dtype=torch.float32) - 0.5).half()
            layer = sharded.ColumnParallelLinear(w, bias, "silu", device=dev, fused_gather=True, max_rows=m)
            ns = layer.weight.shape[0]
            y = layer(a)
            torch.cuda.synchronize()
            # gate: this rank's view of every slice against a torch FP32 reference (sampled rows for large M)
            rows = torch.arange(0, m, max(1, m // 64), device=dev)
            ref = torch.nn.functional.silu(a[rows].float() @ w.float().t() + bias.float())
            err = (y[rows].float() - ref).abs()
            if not bool((err <= 0.02 + 0.002 * ref.abs()).all()):
                raise SystemExit(f"rank {rank}: sharded shape N={n_total} M={m} failed the gate")
            inner = 3 if m >= 1024 else args.inner
            rounds = max(5, min(args.steps, 20))
            call = lambda: layer.gather(a, layer.weight.t(), layer.bias, _native.EPILOGUE_BIAS_SILU)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(inner):
                call()
            host_us = (time.perf_counter() - t0) * 1e6 / inner
            torch.cuda.synchronize()
            hold = max(400.0, 3.0 * inner * host_us)
            token = torch.zeros(1, dtype=torch.float32, device=dev)
            align = lambda: dist.all_reduce(token)
            device_measure({"x": call}, rounds=2, inner=inner, hold_us=hold, align=align)
            dist.barrier()
            raw = device_measure({"x": call}, rounds=rounds, inner=inner, hold_us=hold, align=align)["x"]
            dist.barrier()
            t = torch.tensor([statistics.median(raw)], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t[0]) * 1e3
            single_us = None
            if rank == 0:
                y1 = torch.empty((m, n_total), dtype=torch.float16, device=dev)
                one = lambda: _native.linear(a, w.t(), y1, bias, _native.EPILOGUE_BIAS_SILU)
                device_measure({"x": one}, rounds=2, inner=inner, hold_us=hold)
                single_us = statistics.median(device_measure({"x": one}, rounds=rounds, inner=inner,
                                                             hold_us=hold)["x"]) * 1e3
                del y1
            dist.barrier()
            flops = 2 * m * n_total * k
            rank_bytes = 2 * (m * k + ns * k + m * n_total) + 2 * ns
            row = {"n": n_total, "k": k, "m": m, "n_per_rank": ns, "p50_us": us,
                   "tflops_total": flops / (us * 1e-6) / 1e12,
                   "tensor_frac_per_rank": flops / world / (us * 1e-6) / 1e12 / tensor_peak,
                   "hbm_gbs_per_rank": rank_bytes / (us * 1e-6) / 1e9,
                   "nvlink_bytes_per_rank": 2 * m * ns * (world - 1),
                   "single_gpu_unsharded_us": single_us,
                   "speedup_vs_single_gpu": (single_us / us) if single_us else None}
            out.append(row)
            del layer, y, a
            torch.cuda.empty_cache()
        del w, bias
        torch.cuda.empty_cache()
    return out


def run_native(args) -> int:
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (B200)")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    from gemm_lab_qualification_b200 import _native
    _native.library()  # fail loudly if libglq.so is missing

    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        try:
            res = multi_gpu(args, torch, dist, dev, world, rank)
            if not args.no_sharded_shapes:
                res["sharded_shapes"] = sharded_shapes(args, torch, dist, dev, world, rank)
        finally:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            peak, peak_src = measured_hbm_peak()
            ns, n_total, m = res["shard_rows"], res["n_total"], args.m
            # per-rank bytes: A, this rank's W slice and bias, the full gathered Y written
            rank_bytes = 2 * (m * K_DIM + ns * K_DIM + m * n_total) + 2 * ns
            achieved = rank_bytes / (res["mean_us"] * 1e-6) / 1e9
            line = {"metric": METRIC, "value": res["value"], "unit": "us", "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": res["mean_us"] * 1e-3 * args.inner,
                    "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": DATA,
                    "config": {"workload": f"column-parallel fused linear+bias+SiLU, M={m}, K={K_DIM}, W split along "
                                           f"N: {ns} rows per rank (N={n_total}), all-gather fused into the "
                                           "kernel epilogue (peer stores over NVLink + epoch handshake)",
                               "m": m, "n": n_total, "k": K_DIM, "n_per_rank": ns,
                               "parallelism": f"tp{world} (N-sharded, weak scaling)",
                               "timing": f"CUDA events around {args.inner} back-to-back layer calls behind a GPU "
                                         "hold, the ranks' streams lined up by a one-element all-reduce before "
                                         "each sample, p50 of span/inner, max over ranks",
                               "l2": f"inputs larger than L2: {res['copies']} rotating W-slice copies per rank"},
                    "impl": "native", "gpu_launches": res["gpu_launches"], "clocks": res["clocks"],
                    "local_path": list(res["path"]),
                    "nccl_allgather_comparator_us": res["nccl_us"],
                    "host_enqueue_us_per_call": res["host_us"], "gpu_hold_us": res["hold_us"],
                    "e2e": {"value": res["e2e_us"], "unit": "us", "h2d_bytes_per_step": res["h2d"],
                            "d2h_bytes_per_step": res["d2h"],
                            "note": "per rank: pinned host A, W slice, bias in; gathered Y out; max over ranks"},
                    "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                                 "frac": achieved / peak, "traffic": None, "peak_source": peak_src,
                                 "nvlink_bytes_per_rank": 2 * m * ns * (world - 1),
                                 "nvlink_time_us_at_770_gbs": 2 * m * ns * (world - 1) / 770e9 * 1e6,
                                 "note": "per-rank HBM bytes (A, W slice, bias, gathered Y) over the mean layer "
                                         "call; the NVLink leg (this rank's slice to every peer) is the smaller "
                                         "bound at these sizes"}}
            if "sharded_shapes" in res:
                line["sharded_shapes"] = {
                    "workload": "column-parallel configs: fused linear+bias+SiLU, W [N, K] split along N "
                                "over the ranks (strong scaling), all-gather fused into the kernel; device-"
                                "generator seed-7 uniform inputs; p50 of back-to-back calls, max over ranks; "
                                "tensor_frac against bf16_tflops_sustained of MEASURED_PEAKS.json",
                    "rows": res["sharded_shapes"]}
            print(json.dumps(line), flush=True)
        return 0

    res = single_gpu(args, torch, dev)
    line = {"metric": METRIC, "value": res["value"], "unit": "us", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": DATA,
            "config": {"workload": f"fused linear+bias+SiLU y=SiLU(A W^T + b), value at M={args.m}; step = "
                                   f"M in {list(SWEEP_M)} x {{fused, plain}}, {args.inner} back-to-back calls each, "
                                   f"N=K=4096, W [N,K] K-contiguous",
                       "timing": f"CUDA events around {args.inner} back-to-back calls behind a GPU hold, p50 of "
                                 f"span/{args.inner}",
                       "m": args.m, "n": N_DIM, "k": K_DIM, "parallelism": "single GPU",
                       "l2": f"inputs larger than L2: {res['copies']} rotating W copies "
                             f"({res['copies'] * 32} MiB) > L2 {res['l2_bytes'] / 2**20:.0f} MiB"},
            "impl": "native", "roofline": res["roofline"], "gpu_launches": res["gpu_launches"],
            "clocks": res["clocks"], "sweep": res["sweep"], "mlp_shapes": res["mlp_shapes"]}
    if not args.no_probes:
        line["probes"] = probe_timings(args, torch, dev)
    if not args.no_e2e:
        e2e = e2e_public_api(args, torch, dev, rounds=max(10, min(args.steps, 50)))
        line["e2e"] = e2e["all_inputs"]
        line["e2e_resident_weights"] = e2e["resident_weights"]
    if not args.no_cpu_baseline:
        times, info = cpu_fragment_timings(args.m, args.cpu_seconds, 100000)
        line["cpu_baseline"] = {"value": statistics.median(times), "unit": "us", "cores": info["cores"],
                                "kind": "port", "sample": info["sample"],
                                "reference_full_call_us": info["reference_full_call_us"]}
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_native(args)


if __name__ == "__main__":
    sys.exit(main())
