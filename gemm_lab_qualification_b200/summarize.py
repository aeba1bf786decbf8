"""Markdown report of B200 measurements: the native suite and bench.py.

The reference renders its results page from a run directory
(scripts/summarize.py:4-76; for the GEMM project the native table is at
:25-30: per workload the cuBLASLt, unsplit and split-K medians and the
cuBLASLt / split-K ratio, each the median of three shuffled process-round
medians).  This renderer keeps that table and its statistic and adds what a
memory-bound B200 row needs: the path the library chose, GB/s of the
algorithmic bytes, and the fraction of the measured HBM copy bandwidth, for
the steady (warm-L2) and cold cache modes separately.  With a bench.py JSON
line it also renders the per-M sweep (device-resident, rotating weights),
the MLP shapes, the timed boundary and split-K probes and the end-to-end
(host buffers) number.

``python -m gemm_lab_qualification_b200.summarize suite.json [--bench
bench.json] [--peaks MEASURED_PEAKS.json] --output report.md``
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

FALLBACK_HBM_GBS = 6650.0
IMPL_ORDER = ("cublaslt", "glq", "glq_splitk", "glq_wnk")


def hbm_peak(peaks: dict | None) -> tuple[float, str]:
    """The roofline denominator and how it was obtained."""
    if peaks and peaks.get("hbm_gbs"):
        return float(peaks["hbm_gbs"]), "of measured"
    return FALLBACK_HBM_GBS, "of fallback"


def suite_medians(suite: dict) -> dict:
    """(case, cache, impl) -> {us, gbs, path, rounds}: median over rounds of each round's p50."""
    groups: dict = {}
    for row in suite["results"]:
        rec = row["record"]
        key = (row["case"], row.get("cache", rec["benchmark"].get("cache_mode", "steady")), rec["implementation"]["name"])
        g = groups.setdefault(key, {"us": [], "bytes": rec["benchmark"].get("algorithmic_bytes"), "path": None})
        g["us"].append(rec["benchmark"]["latency_ms"]["p50"] * 1000.0)
        impl = rec["implementation"]
        if impl.get("path"):
            g["path"] = f"{impl['path']}/{impl.get('split_k', 1)}"
        if g["bytes"] is None:
            w = rec["workload"]
            size = 4 if w["input_dtype"] in ("fp32", "float32") else 2
            g["bytes"] = size * (w["m"] * w["k"] + w["k"] * w["n"] + w["m"] * w["n"])
    out = {}
    for key, g in groups.items():
        us = statistics.median(g["us"])
        out[key] = {"us": us, "gbs": g["bytes"] / (us * 1e-6) / 1e9, "path": g["path"], "rounds": len(g["us"])}
    return out


def _fmt(x: float | None, spec: str = ".2f") -> str:
    return "—" if x is None else format(x, spec)


def render_suite(suite: dict, peaks: dict | None = None) -> list[str]:
    peak, source = hbm_peak(peaks)
    med = suite_medians(suite)
    cases = list(dict.fromkeys(row["case"] for row in suite["results"]))
    caches = list(dict.fromkeys(row.get("cache", "steady") for row in suite["results"]))
    impls = [i for i in IMPL_ORDER if any(k[2] == i for k in med)]
    ours = [i for i in impls if i != "cublaslt"]
    env = suite.get("environment", {})
    gpu = env.get("gpu", {}).get("stdout", "").strip().splitlines()
    lines = ["## Native suite (`gemm_bench`, one process per measurement)", "",
             f"Protocol: {suite.get('protocol', '')}.", "",
             f"GPU: `{gpu[1] if len(gpu) > 1 else 'unknown'}`. Source digest `{env.get('source_digest', '?')[:16]}`, "
             f"binary sha256 `{suite.get('binary_sha256', '?')[:16]}`, seed {suite.get('seed')}.", ""]
    for cache in caches:
        title = {"steady": "steady (warm L2: the same operands every call)",
                 "cold": "cold (L2 overwritten and stream synchronised before each single-call sample)"}.get(cache, cache)
        lines += [f"### Cache mode: {title}", "",
                  "| Workload | " + " | ".join(f"{i} µs" for i in impls) + " | best glq | path | GB/s | "
                  f"HBM frac ({source}) | cuBLASLt / best glq |",
                  "|---|" + "---:|" * len(impls) + "---|---|---:|---:|---:|"]
        for case in cases:
            cells = [med.get((case, cache, i)) for i in impls]
            if all(c is None for c in cells):
                continue
            mine = [(med[(case, cache, i)]["us"], i) for i in ours if (case, cache, i) in med]
            best = min(mine) if mine else None
            b = med[(case, cache, best[1])] if best else None
            vendor = med.get((case, cache, "cublaslt"))
            ratio = vendor["us"] / b["us"] if vendor and b else None
            lines.append(f"| {case} | " + " | ".join(_fmt(c and c["us"]) for c in cells) +
                         f" | {best[1] if best else '—'} | {b['path'] if b and b['path'] else '—'} | "
                         f"{_fmt(b and b['gbs'], '.0f')} | {_fmt(b and b['gbs'] / peak, '.3f')} | "
                         f"{_fmt(ratio, '.3f')}{'×' if ratio else ''} |")
        lines.append("")
    lines += ["Each cell is the median over the rounds of that round's p50 (as the reference's report). GB/s counts "
              "the algorithmic bytes 2(MK + KN + MN) once per call; in steady mode the operands of these shapes fit in "
              "L2, so steady GB/s can exceed the HBM figure, and the HBM fraction is meaningful in cold mode only. "
              "Cold single-call samples include the launch gap after the synchronise, as in the reference's CLI.", ""]
    return lines


def render_bench(bench: dict) -> list[str]:
    roof = bench.get("roofline", {})
    lines = ["## bench.py (device-resident inputs, rotating weight copies larger than L2)", "",
             f"Headline: `{bench['metric']}` = **{bench['value']:.2f} {bench['unit']}** "
             f"(roofline {roof.get('frac', 0):.3f} of {roof.get('peak', 0):.0f} {roof.get('unit', '')}, "
             f"{roof.get('kernel', '')}).", ""]
    sweep = bench.get("sweep")
    if sweep:
        items = sweep.items() if isinstance(sweep, dict) else sweep
        lines += ["| M | path | fused p50 µs | GB/s | HBM frac | plain p50 µs | cuBLASLt fused µs | cuBLASLt plain µs | "
                  "fused, lab protocol µs | torch fragment, lab protocol µs |",
                  "|---:|---|---:|---:|---:|---:|---:|---:|---:|---:|"]
        for m, r in items:
            lines.append(f"| {m} | {r['path']}/{r['split']} | {r['fused_p50_us']:.2f} | {r['fused_gbs']:.0f} | "
                         f"{r['fused_frac']:.3f} | {r['plain_p50_us']:.2f} | {_fmt(r.get('cublas_fused_p50_us'))} | "
                         f"{_fmt(r.get('cublas_plain_p50_us'))} | {_fmt(r.get('fused_lab_protocol_p50_us'))} | "
                         f"{_fmt(r.get('torch_fragment_lab_protocol_p50_us'))} |")
        lines.append("")
    mlp = bench.get("mlp_shapes")
    if mlp:
        lines += ["| MLP shape (M×N×K) | path | fused p50 µs | GB/s | cuBLASLt fused µs |", "|---|---|---:|---:|---:|"]
        for r in mlp:
            path = r["path"] if isinstance(r["path"], str) else f"{r['path'][0]}/{r['path'][1]}"
            lines.append(f"| {r['m']}×{r['n']}×{r['k']} | {path} | {r['fused_p50_us']:.2f} | {r['gbs']:.0f} | "
                         f"{_fmt(r.get('cublas_fused_p50_us'))} |")
        lines.append("")
    probes = bench.get("probes")
    if probes:
        lines += [f"Boundary probes ({probes['protocol']}):", "",
                  "| probe | M×N×K | layout | path | p50 µs | GB/s | HBM frac |", "|---|---|---|---|---:|---:|---:|"]
        for r in probes["boundary"]:
            lines.append(f"| {r['id']} | {r['m']}×{r['n']}×{r['k']} | {r['layout']} | {r['path']}/{r['split']} | "
                         f"{r['p50_us']:.2f} | {_fmt(r['gbs'], '.0f')} | {_fmt(r['frac'], '.3f')} |")
        lines += ["", "| split probe | path | p50 µs | GB/s | HBM frac | FP32 partials |",
                  "|---|---|---:|---:|---:|---:|"]
        for r in probes["split"]:
            lines.append(f"| M={r['m']} S={r['split']} | {r['path']}/{r['reported_split']} | {r['p50_us']:.2f} | "
                         f"{r['gbs']:.0f} | {r['frac']:.3f} | {r['partial_bytes'] / 2**10:.0f} KiB |")
        lines.append("")
    e2e, cpu = bench.get("e2e"), bench.get("cpu_baseline")
    if e2e:
        lines += [f"End to end through the operator API with host buffers: {e2e['value']:.1f} {e2e['unit']} per step "
                  f"({e2e['h2d_bytes_per_step']} B host to device, {e2e['d2h_bytes_per_step']} B back).", ""]
    if cpu:
        lines += [f"CPU baseline ({cpu['kind']}, {cpu['cores']} cores): {cpu['value']:.1f} {cpu['unit']} "
                  f"({cpu['sample']}).", ""]
    clocks = bench.get("clocks")
    if clocks:
        lines += [f"Clocks during the timed region: median {clocks['sm_mhz']:.0f} of {clocks['sm_max_mhz']:.0f} MHz, "
                  f"reasons {clocks['reasons'] or 'none'}.", ""]
    return lines


def render(suite: dict | None = None, bench: dict | None = None, peaks: dict | None = None) -> str:
    lines = ["# B200 measurements", ""]
    if suite is not None:
        lines += render_suite(suite, peaks)
    if bench is not None:
        lines += render_bench(bench)
    return "\n".join(lines).rstrip() + "\n"


def _load_json_line(path: str) -> dict:
    text = Path(path).read_text().strip()
    try:
        return json.loads(text)
    except json.JSONDecodeError:
        return json.loads(text.splitlines()[-1])


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("suite", nargs="?", help="native_suite JSON")
    p.add_argument("--bench", help="bench.py output (its last line is the JSON record)")
    p.add_argument("--peaks", help="MEASURED_PEAKS.json (roofline denominators)")
    p.add_argument("--output", help="Markdown file (default: stdout)")
    a = p.parse_args(argv)
    if a.suite is None and a.bench is None:
        p.error("give a suite JSON, --bench, or both")
    text = render(_load_json_line(a.suite) if a.suite else None, _load_json_line(a.bench) if a.bench else None,
                  json.loads(Path(a.peaks).read_text()) if a.peaks else None)
    if a.output:
        Path(a.output).write_text(text)
    else:
        sys.stdout.write(text)
    return 0


if __name__ == "__main__":
    sys.exit(main())
