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


# ------------------------------------------------------------- several GPUs
class FakeProc:
    def __init__(self, returncode, hang=False):
        self.returncode = returncode
        self.hang = hang
        self.killed = False

    def wait(self, timeout=None):
        if self.hang and not self.killed:
            raise subprocess.TimeoutExpired("child", timeout)
        return self.returncode

    def kill(self):
        self.killed = True


class FakePopen:
    """Concurrent children: writes each device's document; behaviour per (metric, device)."""

    def __init__(self, behaviour=None, scale=None):
        self.behaviour = behaviour or {}
        self.scale = scale or {}
        self.calls = []

    def __call__(self, command, cwd, stdout, stderr):
        output = Path(command[command.index("--output") + 1])
        device = int(command[command.index("--device") + 1])
        self.calls.append((device, command))
        key = output.name.split(".gpu")[0]
        metric = next(m for m in METRICS if m.key == key)
        action = self.behaviour.get((key, device), "ok")
        if action == "hang":
            return FakeProc(None, hang=True)
        if action == "crash":
            return FakeProc(2)
        if action == "unsupported":
            output.write_text(json.dumps({"status": "unsupported", "reason": "nope"}))
            return FakeProc(0)
        document = ok_document(metric)
        factor = self.scale.get(device, 1.0)
        for row in document["results"]:
            for field in ("peak_gbps", "gbps", "peak_teraops_per_second",
                          "median_teraops_per_second", "peak_tflops", "tflops"):
                if field in row:
                    row[field] *= factor
        output.write_text(json.dumps(document))
        return FakeProc(0)


def test_multi_gpu_table_aggregates_per_gpu_rows(tmp_path, capsys):
    args = args_for(tmp_path, gpus=2)
    popen = FakePopen(scale={1: 0.5})
    report = bench_suite.run_suite(args, popen=popen)
    assert report["status"] == "complete" and report["n_gpus"] == 2
    assert sorted({device for device, _ in popen.calls}) == [0, 1]
    rows = {r["metric"]: r for r in report["results"]}
    bw = rows["memory_bandwidth"]
    assert bw["status"] == "ok" and bw["value"] == pytest.approx(6400.0 * 1.5)
    assert [sub["device_index"] for sub in bw["per_gpu"]] == [0, 1]
    assert bw["per_gpu"][1]["value"] == pytest.approx(3200.0)
    assert bw["aggregation"]["n_gpus"] == 2 and bw["aggregation"]["per_gpu_value_min"] == 3200.0
    assert rows["memory_capacity"]["value"] == pytest.approx(2 * 183.0)
    assert rows["tensor_bf16"]["median_value"] == pytest.approx(1490.0 * 1.5)
    assert rows["tensor_bf16"]["execution_kind"] == "tensor"
    out = capsys.readouterr().out
    assert "Per GPU:" in out and "GPU 1" in out
    # the table keeps the single-GPU schema: same 17 keys in the same order
    assert [r["metric"] for r in report["results"]] == [m.key for m in METRICS]


def test_multi_gpu_failure_is_reported_per_gpu(tmp_path):
    args = args_for(tmp_path, gpus=2, metrics=["tensor_bf16", "vector_fp32", "tensor_fp4"])
    popen = FakePopen(behaviour={("tensor_bf16", 1): "crash", ("vector_fp32", 0): "hang",
                                 ("tensor_fp4", 0): "unsupported",
                                 ("tensor_fp4", 1): "unsupported"})
    report = bench_suite.run_suite(args, popen=popen)
    rows = {r["metric"]: r for r in report["results"]}
    bf16 = rows["tensor_bf16"]
    assert bf16["status"] == "error" and "GPU 1" in bf16["reason"] and bf16["value"] is None
    assert bf16["partial_measurement"] == {"gpus": 1, "value": 1500.0}
    vec = rows["vector_fp32"]
    assert vec["status"] == "error" and "GPU 0" in vec["reason"]
    assert "Exceeded" in vec["per_gpu"][0]["reason"]
    assert rows["tensor_fp4"]["status"] == "unsupported"
    assert report["status"] == "complete_with_errors"


def test_window_overlap():
    assert bench_suite.window_overlap([(0, 10), (1, 10)]) == pytest.approx(1.0)
    assert bench_suite.window_overlap([(0, 10), (5, 20)]) == pytest.approx(0.5)
    assert bench_suite.window_overlap([(0, 1), (2, 3)]) == 0.0
    assert bench_suite.window_overlap([]) is None
