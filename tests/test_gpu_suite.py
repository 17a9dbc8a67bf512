"""The suite's drivers end to end on the GPU (the 17-row table and its children).

* ``bench_suite --quick`` writes all 17 rows in the contract's order: the
  capacity row equals what CUDA reports, every tensor and vector row was
  measured and validated, vector_fp8 is not_implemented and vector_fp4
  unsupported exactly as in the reference (bench_vector.py:1054-1102), and
  every child document summarizes to the row the suite wrote;
* the bandwidth child at an HBM-sized buffer (not smoke mode) yields an
  eligible copy peak plus the read pattern, after its masked-tail checks,
  with the reference's row fields (bench_bandwidth.py:136-249);
* vector rows carry the audit fields of the reference's inspect_assembly
  (bench_vector.py:772-798);
* tcb_device_query agrees with torch's view of the device.
"""

import json
from pathlib import Path
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def quick_suite(cuda, tmp_path_factory):
    out = tmp_path_factory.mktemp("suite") / "quick.json"
    command = [sys.executable, "-m", "triton_chip_benchmarks_b200.bench_suite", "--device", "0",
               "--quick", "--warmup", "5", "--rep", "10", "--timeout", "300",
               "--output", str(out)]
    proc = subprocess.run(command, cwd=REPO, capture_output=True, text=True, timeout=1800)
    assert out.exists(), proc.stdout[-2000:] + proc.stderr[-2000:]
    return json.loads(out.read_text()), proc


def test_quick_suite_writes_the_17_rows(quick_suite):
    from triton_chip_benchmarks_b200.suite_report import METRICS
    report, proc = quick_suite
    assert report["benchmark"] == "chip_metric_suite" and report["schema_version"] == 1
    assert [row["metric"] for row in report["results"]] == [m.key for m in METRICS]
    status = {row["metric"]: row["status"] for row in report["results"]}
    assert status["vector_fp8"] == "not_implemented"
    assert status["vector_fp4"] == "unsupported"
    assert status["memory_capacity"] == "ok"
    # Smoke mode never yields an HBM-sized copy peak (as in the reference).
    assert status["memory_bandwidth"] == "not_measured"
    errors = {k: v for k, v in status.items() if v == "error"}
    assert not errors, (errors, proc.stdout[-3000:])
    for row in report["results"]:
        if row["group"] in ("Tensor", "Vector") and row["metric"] not in ("vector_fp8",
                                                                        "vector_fp4"):
            assert row["status"] in ("ok", "unverified"), row
            assert row["value"] > 0 and row["smoke_only"] is True, row


def test_capacity_row_is_what_cuda_reports(quick_suite, cuda):
    report, _ = quick_suite
    row = next(r for r in report["results"] if r["metric"] == "memory_capacity")
    total = torch.cuda.get_device_properties(cuda).total_memory
    assert row["capacity_bytes"] == total
    assert row["value"] == pytest.approx(total / 2**30, rel=0, abs=1e-9)


def test_every_child_document_summarizes_to_its_row(quick_suite):
    from triton_chip_benchmarks_b200.suite_report import METRICS, summarize
    report, _ = quick_suite
    for metric, row in zip(METRICS, report["results"]):
        document = json.loads(Path(row["source_json"]).read_text())
        again = summarize(metric, document)
        assert again["status"] == row["status"], metric.key
        assert again.get("value") == row.get("value"), metric.key


def test_vector_rows_carry_the_audit_fields(quick_suite):
    report, _ = quick_suite
    for key in ("vector_bf16", "vector_fp16", "vector_fp32", "vector_fp64", "vector_int8"):
        row = next(r for r in report["results"] if r["metric"] == key)
        document = json.loads(Path(row["source_json"]).read_text())
        measured = [r for r in document["results"] if r.get("status", "ok") == "ok"]
        assert measured, key
        for r in measured:
            assert r["register_spills"] == 0
            assert r["native_arithmetic_verified"] is True
            assert r["ptx_contains_tensor_instructions"] is False
            assert r["assembly_check"].startswith("passed")
            assert r["ptx_arithmetic_instruction"]


def test_bandwidth_child_at_hbm_size(cuda, tmp_path):
    from triton_chip_benchmarks_b200.suite_report import METRICS, summarize
    out = tmp_path / "bandwidth.json"
    command = [sys.executable, "-m", "triton_chip_benchmarks_b200.bench_bandwidth", "--mode",
               "all", "--dtype", "fp32", "--sizes-mib", "1024", "--warmup", "5", "--rep", "20",
               "--output", str(out)]
    proc = subprocess.run(command, cwd=REPO, capture_output=True, text=True, timeout=900)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-2000:]
    assert "masked tails passed" in proc.stdout
    document = json.loads(out.read_text())
    metric = next(m for m in METRICS if m.key == "memory_bandwidth")
    row = summarize(metric, document)
    assert row["status"] == "ok", row
    assert set(row["patterns"]) == {"copy", "read"}
    for r in document["results"]:
        assert r["cache_regime"] == "larger_than_l2" and r["peak_eligible"] is True
        assert r["read_bytes"] == r["buffer_bytes"] == 1024 * 2**20
        if r["pattern"] == "copy":
            assert r["traffic_bytes"] == 2 * r["buffer_bytes"]
            assert r["correctness"].startswith("passed")
    # An HBM-bound copy on B200: well above anything a cache could explain away.
    assert row["value"] > 4000


def test_device_query_matches_torch(cuda, native):
    props = torch.cuda.get_device_properties(cuda)
    mine = native.device_query(0)
    assert mine.sm_count == props.multi_processor_count
    assert mine.total_mem_bytes == props.total_memory
    assert (mine.major, mine.minor) == (props.major, props.minor)
    assert mine.l2_cache_bytes == props.L2_cache_size
    assert mine.name == props.name
    assert 0 < mine.free_mem_bytes <= mine.total_mem_bytes
