"""Native suite driver and report renderer.

CPU: the driver's protocol (shuffled rounds, one child per measurement,
abort on a failing child or a failed correctness gate, the gate check) is
exercised against a stand-in CLI that prints schema-v1 records; the renderer
is checked on hand-made records.  GPU: one round of the real suite on the
decode and tail shapes, rendered.
"""
from __future__ import annotations

import json
import os
import stat
import sys
from pathlib import Path

import pytest

from gemm_lab_qualification_b200 import native_suite, summarize

FAKE_CLI = r'''#!{python}
import json, sys
a = dict(zip(sys.argv[1::2], sys.argv[2::2]))
if a["--impl"] == "{fail_impl}":
    sys.stderr.write("gemm_bench: planted failure\n"); sys.exit(1)
m, n, k = int(a["--m"]), int(a["--n"]), int(a["--k"])
us = {{"cublaslt": 20.0, "glq": 10.0, "glq_splitk": 12.0, "glq_wnk": 11.0}}[a["--impl"]]
if a["--cache"] == "cold":
    us *= 2
with open("{log}", "a") as log:
    log.write(" ".join(sys.argv[1:]) + "\n")
rec = {{"schema_version": 1,
        "implementation": {{"name": a["--impl"], "version": "fake"}},
        "workload": {{"m": m, "n": n, "k": k, "input_dtype": "fp16"}},
        "correctness": {{"passed": a["--impl"] != "{bad_impl}", "reference": "cublas_full"}},
        "benchmark": {{"cache_mode": a["--cache"], "samples": int(a["--samples"]),
                       "latency_ms": {{"p50": us / 1000.0}}, "algorithmic_bytes": 2 * (m * k + k * n + m * n)}}}}
if a["--impl"].startswith("glq"):
    rec["implementation"].update(path="tc_splitk", split_k=8)
print(json.dumps(rec))
'''


def fake_cli(tmp_path: Path, fail_impl: str = "", bad_impl: str = "") -> tuple[Path, Path]:
    log = tmp_path / "calls.log"
    path = tmp_path / "gemm_bench"
    path.write_text(FAKE_CLI.format(python=sys.executable, fail_impl=fail_impl, bad_impl=bad_impl, log=log))
    path.chmod(path.stat().st_mode | stat.S_IEXEC)
    return path, log


SHAPES = [{"id": "decode-m32", "m": 32, "n": 4096, "k": 4096}, {"id": "tail", "m": 17, "n": 257, "k": 131}]


def test_rounds_are_shuffled_and_every_child_recorded(tmp_path):
    cli, log = fake_cli(tmp_path)
    doc = native_suite.run(binary=cli, shapes=SHAPES, samples=5)
    per_round = len(SHAPES) * len(native_suite.IMPLS) * len(native_suite.CACHE_MODES)
    assert len(doc["results"]) == 3 * per_round
    assert doc["status"] == "measured" and doc["seed"] == 1729
    calls = log.read_text().splitlines()
    assert len(calls) == 3 * per_round
    rounds = [calls[i * per_round:(i + 1) * per_round] for i in range(3)]
    assert all(sorted(r) == sorted(rounds[0]) for r in rounds)
    assert rounds[0] != rounds[1] or rounds[1] != rounds[2]
    argv = doc["results"][0]["argv"]
    assert argv[argv.index("--seed") + 1] == "1729" and argv[argv.index("--measurement-seconds") + 1] == "0"
    # Same seed, same order: the protocol is reproducible.
    again = native_suite.run(binary=cli, shapes=SHAPES, samples=5)
    assert [r["argv"] for r in again["results"]] == [r["argv"] for r in doc["results"]]


def test_failing_child_aborts(tmp_path):
    cli, _ = fake_cli(tmp_path, fail_impl="glq_wnk")
    with pytest.raises(RuntimeError, match="planted failure"):
        native_suite.run(binary=cli, shapes=SHAPES[:1], rounds=1)


def test_failed_correctness_aborts(tmp_path):
    cli, _ = fake_cli(tmp_path, bad_impl="glq_splitk")
    with pytest.raises(AssertionError, match="native correctness failed"):
        native_suite.run(binary=cli, shapes=SHAPES[:1], rounds=1)


def test_gate_must_pass_on_these_sources(tmp_path):
    cli, _ = fake_cli(tmp_path)
    gate = tmp_path / "gate.json"
    gate.write_text(json.dumps({"status": "passed", "environment": {"source_digest": "stale"}}))
    with pytest.raises(RuntimeError, match="stale correctness gate"):
        native_suite.run(gate=gate, binary=cli, shapes=SHAPES[:1], rounds=1)
    gate.write_text(json.dumps({"status": "failed", "environment": {"source_digest": native_suite.source_digest()}}))
    with pytest.raises(RuntimeError):
        native_suite.run(gate=gate, binary=cli, shapes=SHAPES[:1], rounds=1)
    gate.write_text(json.dumps({"status": "passed", "environment": {"source_digest": native_suite.source_digest()}}))
    doc = native_suite.run(gate=gate, binary=cli, shapes=SHAPES[:1], rounds=1, cache_modes=("steady",))
    assert doc["gate"] == str(gate) and len(doc["results"]) == len(native_suite.IMPLS)


def test_save_is_atomic_and_rejects_nan(tmp_path):
    target = tmp_path / "out" / "suite.json"
    native_suite.save(target, {"a": 1})
    with pytest.raises(ValueError):
        native_suite.save(target, {"a": float("nan")})
    assert json.loads(target.read_text()) == {"a": 1}
    assert os.listdir(target.parent) == ["suite.json"]


def test_report_medians_gbs_and_ratio(tmp_path):
    cli, _ = fake_cli(tmp_path)
    doc = native_suite.run(binary=cli, shapes=SHAPES, samples=5)
    med = summarize.suite_medians(doc)
    cell = med[("decode-m32", "cold", "glq")]
    assert cell["us"] == pytest.approx(20.0) and cell["rounds"] == 3 and cell["path"] == "tc_splitk/8"
    nbytes = 2 * (32 * 4096 + 4096 * 4096 + 32 * 4096)
    assert cell["gbs"] == pytest.approx(nbytes / 20e-6 / 1e9)
    text = summarize.render(doc, peaks={"hbm_gbs": 6538.0})
    cold = text.split("Cache mode: cold")[1]
    row = next(line for line in cold.splitlines() if line.startswith("| decode-m32"))
    assert row.startswith("| decode-m32 | 40.00 | 20.00 | 24.00 | 22.00 |") and "2.000×" in row
    assert "| glq |" in row and f"| {nbytes / 20e-6 / 1e9 / 6538.0:.3f} |" in row
    assert "of measured" in text and "Cache mode: cold" in text and "Cache mode: steady" in text
    assert "of fallback" in summarize.render(doc)


def test_report_of_bench_line():
    bench = {"metric": "p50", "value": 10.0, "unit": "us",
             "roofline": {"frac": 0.52, "peak": 6538.0, "unit": "GB/s", "kernel": "tc_linear"},
             "sweep": {"32": {"path": "tc_splitk", "split": 8, "fused_p50_us": 10.0, "fused_gbs": 3400.0,
                              "fused_frac": 0.52, "plain_p50_us": 9.8, "cublas_fused_p50_us": 20.0}},
             "mlp_shapes": [{"m": 32, "n": 11008, "k": 4096, "path": ["tc_splitk", 3], "fused_p50_us": 22.5,
                             "gbs": 4041.0, "cublas_fused_p50_us": 25.0}],
             "e2e": {"value": 675.5, "unit": "us", "h2d_bytes_per_step": 10, "d2h_bytes_per_step": 2},
             "cpu_baseline": {"value": 3201.8, "unit": "us", "cores": 16, "kind": "port", "sample": "s"},
             "clocks": {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []},
             "probes": {"protocol": "p",
                        "boundary": [{"id": "zero-m", "m": 0, "n": 4096, "k": 4096, "layout": "w_nk", "path": "empty",
                                      "split": 1, "p50_us": 0.0, "gbs": None, "frac": None},
                                     {"id": "tail-k", "m": 32, "n": 4096, "k": 4090, "layout": "w_nk",
                                      "path": "repacked", "split": 8, "p50_us": 25.0, "gbs": 1340.0, "frac": 0.2}],
                        "split": [{"m": 8, "split": 4, "path": "tc_splitk", "reported_split": 4, "p50_us": 11.0,
                                   "gbs": 3060.0, "frac": 0.468, "partial_bytes": 4 * 8 * 4096 * 4}]}}
    text = summarize.render(bench=bench)
    assert "| zero-m | 0×4096×4096 | w_nk | empty/1 | 0.00 | — | — |" in text
    assert "| tail-k | 32×4096×4090 | w_nk | repacked/8 | 25.00 | 1340 | 0.200 |" in text
    assert "| M=8 S=4 | tc_splitk/4 | 11.00 | 3060 | 0.468 | 512 KiB |" in text
    assert "| 32 | tc_splitk/8 | 10.00 | 3400 | 0.520 | 9.80 | 20.00 |" in text
    assert "| 32×11008×4096 | tc_splitk/3 | 22.50 | 4041 | 25.00 |" in text
    assert "675.5 us" in text and "reasons none" in text


@pytest.mark.gpu
def test_suite_on_the_device(cuda_device, tmp_path):
    shapes = [s for s in native_suite.MANIFEST["benchmark"] if s["id"] in ("decode-m32", "tail")]
    doc = native_suite.run(shapes=shapes, rounds=1, warmup=2, samples=3)
    assert len(doc["results"]) == len(shapes) * len(native_suite.IMPLS) * len(native_suite.CACHE_MODES)
    for row in doc["results"]:
        bench = row["record"]["benchmark"]
        assert bench["cache_mode"] == row["cache"] and bench["gbs_p50"] > 0
        assert bench["algorithmic_bytes"] > 0
    target = tmp_path / "suite.json"
    native_suite.save(target, doc)
    text = summarize.render(json.loads(target.read_text()))
    assert "| decode-m32 |" in text and "| tail |" in text


def test_command_lines(tmp_path, capsys):
    cli, _ = fake_cli(tmp_path)
    suite = tmp_path / "suite.json"
    assert native_suite.main(["--output", str(suite), "--binary", str(cli), "--rounds", "1", "--impls",
                              "cublaslt,glq", "--cache", "steady"]) == 0
    doc = json.loads(suite.read_text())
    assert {r["record"]["implementation"]["name"] for r in doc["results"]} == {"cublaslt", "glq"}
    assert len(doc["results"]) == 2 * len(native_suite.MANIFEST["benchmark"])
    report = tmp_path / "report.md"
    assert summarize.main([str(suite), "--output", str(report)]) == 0
    assert "| decode-m32 |" in report.read_text() and "Cache mode: cold" not in report.read_text()
    assert summarize.main([str(suite)]) == 0
    assert "# B200 measurements" in capsys.readouterr().out
    with pytest.raises(SystemExit):
        summarize.main([])
