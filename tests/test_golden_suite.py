"""Suite table contract and timing policy pinned to the reference's own outputs (CPU)."""

import json
import math

import pytest

from conftest import GOLDEN
from fake_device import SCENARIOS, FakeDeviceAPI, make_args
from triton_chip_benchmarks_b200 import runtime, suite_report

SUITE = json.loads((GOLDEN / "suite.json").read_text())
TIMING = json.loads((GOLDEN / "timing.json").read_text())
BANDWIDTH = json.loads((GOLDEN / "bandwidth.json").read_text())


def test_metric_table_is_identical():
    assert [[m.key, m.group, m.precision, m.unit] for m in suite_report.METRICS] == \
        SUITE["metrics"]
    assert len(suite_report.METRICS) == 17
    assert [suite_report.empty_metric(m) for m in suite_report.METRICS] == SUITE["empty"]


@pytest.mark.parametrize("index", range(len(SUITE["cases"])))
def test_summarize_matches_reference(index):
    case = SUITE["cases"][index]
    metric = {m.key: m for m in suite_report.METRICS}[case["metric"]]
    assert suite_report.summarize(metric, case["document"]) == case["result"]


def test_format_table_matches_reference():
    assert suite_report.format_table(SUITE["table_input"]) == SUITE["table"]


NUMERIC = ("median_ms", "p20_ms", "p80_ms", "min_ms", "max_ms", "launches_per_batch",
           "sample_count", "measured_total_ms", "calibration_launches",
           "minimum_resolved_batch_ms")


@pytest.mark.parametrize("name", sorted(SCENARIOS))
def test_measure_matches_reference_policy(name, capsys):
    spec, golden = SCENARIOS[name], TIMING[name]
    api = FakeDeviceAPI(**spec["api"])
    args = make_args(**spec["args"])
    if "error" in golden:
        with pytest.raises(RuntimeError):
            runtime.measure(api.launch, args, api=api)
        assert api.launches == golden["launches"] and api.replays == golden["replays"]
        return
    result = runtime.measure(api.launch, args, api=api)
    expected = golden["result"]
    for key in NUMERIC:
        assert math.isclose(result[key], expected[key], rel_tol=1e-12, abs_tol=1e-12), key
    assert result["samples_ms_per_launch"] == pytest.approx(expected["samples_ms_per_launch"])
    assert result["batch_samples_ms"] == pytest.approx(expected["batch_samples_ms"])
    assert result["timing_method"] == expected["timing_method"]
    assert result["timing_requested"] == expected["timing_requested"]
    assert (result["timing_fallback_reason"] is None) == (expected["timing_fallback_reason"]
                                                          is None)
    assert (result["graph_api"] is None) == (expected["graph_api"] is None)
    assert set(result) == set(expected)
    assert api.launches == golden["launches"] and api.replays == golden["replays"]
    assert api.now_ms == pytest.approx(golden["final_clock_ms"])


def test_measure_never_uses_host_clock(monkeypatch):
    import time

    def forbidden(*a, **k):
        raise AssertionError("host clock used for device timing")

    monkeypatch.setattr(time, "perf_counter", forbidden)
    monkeypatch.setattr(time, "monotonic", forbidden)
    monkeypatch.setattr(time, "time", forbidden)
    api = FakeDeviceAPI(kernel_ms=0.3)
    result = runtime.measure(api.launch, make_args(), api=api)
    assert result["min_ms"] == pytest.approx(0.3)


def test_read_check_verdicts():
    import torch

    from oracle import native as oracle_native
    from triton_chip_benchmarks_b200.validation import check_read
    for case in BANDWIDTH:
        src = torch.tensor(case["src"], dtype=torch.float32)
        sink = torch.tensor(case["sink"], dtype=torch.float32)
        try:
            check_read(src, sink, case["block"])
            accepted = True
        except AssertionError:
            accepted = False
        assert accepted == case["accepted"], case["case"]
        sums, abs_sums = oracle_native.block_sums(src.numpy(), case["block"])
        import numpy as np
        tol = abs_sums * 2 * np.finfo(np.float32).eps * max(1, math.log2(case["block"])) + 1e-6
        assert bool(np.all(np.abs(sink.double().numpy() - sums) <= tol)) == case["accepted"]
