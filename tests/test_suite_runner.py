"""Suite runner: child isolation, stale output, timeouts, checkpoints (CPU, faked children).

Mirrors the reference's runner tests (tests/test_suite.py:163-247): children
are replaced by a fake subprocess runner that writes chosen JSON documents,
exits non-zero, times out or writes nothing.
"""

import json
import subprocess
from pathlib import Path
from types import SimpleNamespace

import pytest

from triton_chip_benchmarks_b200 import bench_suite
from triton_chip_benchmarks_b200.suite_report import METRICS


def args_for(tmp_path, **kw):
    parser = bench_suite.build_parser()
    args = parser.parse_args(["--output", str(tmp_path / "table.json")])
    for key, value in kw.items():
        setattr(args, key, value)
    return args


def ok_document(metric):
    if metric.key == "memory_capacity":
        return {"status": "ok", "device": {"total_memory_bytes": 183 * 2**30}, "results": []}
    if metric.key == "memory_bandwidth":
        return {"status": "ok", "device": {"device_name": "fake"}, "results": [
            {"pattern": "copy", "peak_gbps": 6400.0, "gbps": 6300.0, "peak_eligible": True}]}
    if metric.group == "Tensor":
        return {"status": "ok", "device": {}, "results": [
            {"status": "ok", "peak_teraops_per_second": 1500.0,
             "median_teraops_per_second": 1490.0,
             "compiled": {"execution_kind": "tensor", "native_tensor_verified": True,
                          "instruction_precision_verified": True}}]}
    return {"status": "ok", "device": {}, "results": [
        {"status": "ok", "peak_tflops": 70.0, "tflops": 69.0, "peak_tops": 70.0, "tops": 69.0,
         "native_arithmetic_verified": True}]}


class FakeRunner:
    def __init__(self, behaviour):
        self.behaviour = behaviour
        self.calls = []

    def __call__(self, command, cwd, stdout, stderr, timeout, check):
        output = Path(command[command.index("--output") + 1])
        module = command[command.index("-m") + 1]
        self.calls.append((module, command))
        metric = next(m for m in METRICS if output.stem == m.key)
        action = self.behaviour.get(metric.key, "ok")
        if action == "timeout":
            raise subprocess.TimeoutExpired(command, timeout)
        if action == "nothing":
            return SimpleNamespace(returncode=1)
        if action == "garbage":
            output.write_text("{not json")
            return SimpleNamespace(returncode=0)
        if action == "crash_after_write":
            output.write_text(json.dumps(ok_document(metric)))
            return SimpleNamespace(returncode=3)
        if action == "unsupported_exit":
            output.write_text(json.dumps({"status": "unsupported", "reason": "nope"}))
            return SimpleNamespace(returncode=1)
        output.write_text(json.dumps(ok_document(metric)))
        return SimpleNamespace(returncode=0)


def test_commands_use_package_children(tmp_path):
    args = args_for(tmp_path)
    commands = {m.key: bench_suite.metric_command(m, args, tmp_path / f"{m.key}.json")
                for m in METRICS}
    assert commands["memory_capacity"][3].endswith("bench_suite") and \
        "--probe-device" in commands["memory_capacity"]
    assert commands["memory_bandwidth"][3].endswith("bench_bandwidth")
    tf32 = commands["tensor_tf32"]
    assert tf32[tf32.index("--dtype") + 1] == "fp32" and \
        tf32[tf32.index("--input-precision") + 1] == "tf32"
    fp32 = commands["tensor_fp32"]
    assert fp32[fp32.index("--input-precision") + 1] == "ieee"
    assert commands["vector_fp8"][3].endswith("bench_vector")


def test_full_table_all_ok(tmp_path, capsys):
    runner = FakeRunner({})
    report = bench_suite.run_suite(args_for(tmp_path), runner)
    assert report["status"] == "complete"
    assert [r["metric"] for r in report["results"]] == [m.key for m in METRICS]
    assert all(r["status"] == "ok" for r in report["results"])
    saved = json.loads((tmp_path / "table.json").read_text())
    assert saved["schema_version"] == 1 and saved["benchmark"] == "chip_metric_suite"
    assert "Metric" in capsys.readouterr().out


def test_failures_are_isolated(tmp_path):
    runner = FakeRunner({"tensor_fp8": "timeout", "vector_fp16": "nothing",
                         "vector_bf16": "garbage", "tensor_bf16": "crash_after_write",
                         "vector_fp4": "unsupported_exit"})
    report = bench_suite.run_suite(args_for(tmp_path), runner)
    by = {r["metric"]: r for r in report["results"]}
    assert report["status"] == "complete_with_errors"
    assert by["tensor_fp8"]["status"] == "error" and "Exceeded" in by["tensor_fp8"]["reason"]
    assert by["vector_fp16"]["status"] == "error"
    assert "Invalid benchmark JSON" in by["vector_bf16"]["reason"]
    assert by["tensor_bf16"]["status"] == "error"
    assert by["tensor_bf16"]["partial_measurement"]["status"] == "ok"
    assert by["vector_fp4"]["status"] == "unsupported"
    assert by["tensor_fp16"]["status"] == "ok"


def test_stale_output_is_removed(tmp_path):
    directory = tmp_path / "table_runs"
    directory.mkdir()
    stale = directory / "tensor_fp16.json"
    stale.write_text(json.dumps({"status": "ok", "results": [
        {"status": "ok", "peak_teraops_per_second": 9.0, "median_teraops_per_second": 9.0}]}))
    runner = FakeRunner({"tensor_fp16": "nothing"})
    report = bench_suite.run_suite(args_for(tmp_path), runner)
    by = {r["metric"]: r for r in report["results"]}
    assert by["tensor_fp16"]["status"] == "error"
    assert not stale.exists()


def test_checkpoint_after_every_metric(tmp_path):
    seen = []
    inner = FakeRunner({})

    def runner(command, **kw):
        table = tmp_path / "table.json"
        if table.exists():
            seen.append(sum(r["status"] != "pending" for r in json.loads(table.read_text())
                            ["results"]))
        return inner(command, **kw)

    bench_suite.run_suite(args_for(tmp_path), runner)
    assert seen == list(range(len(METRICS)))


def test_quick_marks_smoke(tmp_path):
    report = bench_suite.run_suite(args_for(tmp_path, quick=True), FakeRunner({}))
    by = {r["metric"]: r for r in report["results"]}
    assert by["tensor_bf16"].get("smoke_only") is True
    assert not by["memory_bandwidth"].get("smoke_only")
