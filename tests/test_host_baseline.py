"""Host baselines (the reference's CPU validation paths, timed): shape and checks."""

from triton_chip_benchmarks_b200 import host_baseline


def test_quick_run_reports_every_case_with_positive_rates():
    document = host_baseline.run_all(quick=True)
    cases = [(row["case"], row.get("dtype")) for row in document["rows"]]
    assert cases[0] == ("tile", None)
    assert {("tensor", d) for d in ("bf16", "fp32", "fp64", "int8")} <= set(cases)
    assert {("vector", d) for d in ("fp32", "fp64")} <= set(cases)
    for row in document["rows"]:
        assert row["gflops"] > 0 and row["best_s"] <= row["median_s"]
    assert document["threads"] >= 1 and document["cpu_count"] >= 1


def test_tile_case_counts_the_baseline_operations():
    row = host_baseline.tile_baseline(repeats=1)
    assert row["operations"] == 2 * 128 * 128 * 64 * 4
