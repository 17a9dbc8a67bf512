"""The 17-row chip metric table and the summary of each child's JSON document.

This keeps the reference suite's table contract (suite_report.py:15-170):
the same (key, group, precision, unit) rows in the same order, the same
status vocabulary (ok, unverified, unsupported, not_implemented, error,
not_measured, unavailable, pending), peak = best valid row's minimum-time
rate with the median from the same configuration, and for memory bandwidth
the best HBM-sized copy row with copy/read kept under ``patterns``.
Missing measurements are never reported as zero.
"""

from __future__ import annotations

from dataclasses import dataclass
import math


@dataclass(frozen=True)
class Metric:
    key: str
    group: str
    precision: str | None
    unit: str


def _unit(dtype: str) -> str:
    return "TOP/s" if dtype == "int8" else "TFLOP/s"


METRICS = (
    Metric("memory_capacity", "Memory", None, "GiB"),
    Metric("memory_bandwidth", "Memory", None, "GB/s"),
    *(Metric(f"tensor_{d}", "Tensor", d, _unit(d))
      for d in ("bf16", "fp16", "fp32", "tf32", "int8", "fp64", "fp8", "fp4")),
    *(Metric(f"vector_{d}", "Vector", d, _unit(d))
      for d in ("bf16", "fp16", "fp32", "int8", "fp64", "fp8", "fp4")),
)

_DETAIL_KEYS = (
    "execution_kind", "native_tensor_verified", "native_arithmetic_verified",
    "instruction_precision_verified", "precision_verified", "assembly_check",
    "assembly_audit", "assembly_audit_note", "arithmetic_dtype", "includes_unpacking",
    "input_storage_dtype", "accumulator_dtype", "output_dtype", "operation",
    "measurement_kind", "timing_method", "timing_fallback_reason",
)
_CONFIG_KEYS = ("config", "block_size", "num_warps", "unroll", "blocks_per_sm", "blocks",
                "iterations", "pattern", "buffer_mib", "cache_regime", "peak_eligible")


def empty_metric(metric: Metric, status: str = "pending", reason: str | None = None) -> dict:
    result = {"metric": metric.key, "group": metric.group, "precision": metric.precision,
              "unit": metric.unit, "status": status, "value": None, "median_value": None}
    if reason:
        result["reason"] = reason
    return result


def _is_rate(value) -> bool:
    return (isinstance(value, (int, float)) and not isinstance(value, bool)
            and math.isfinite(value) and value > 0)


def _rates(metric: Metric, row: dict):
    """(peak, median) of one result row in the metric's unit."""
    if metric.key == "memory_bandwidth":
        return row.get("peak_gbps"), row.get("gbps")
    suffix = "tops" if metric.precision == "int8" else "tflops"
    return (_first_set(row, "peak_teraops_per_second", f"peak_{suffix}"),
            _first_set(row, "median_teraops_per_second", suffix))


def _first_set(row: dict, *keys):
    """The first of `keys` whose value in `row` is not None."""
    return next((row[key] for key in keys if row.get(key) is not None), None)


def _has_rates(metric: Metric, row) -> bool:
    return (isinstance(row, dict) and row.get("status", "ok") == "ok"
            and all(_is_rate(v) for v in _rates(metric, row)))


def _peak_of(metric: Metric):
    return lambda row: _rates(metric, row)[0]


def _row_details(metric: Metric, row: dict) -> dict:
    """Value, median, audit fields (the row's own over its compiled record) and
    the configuration that produced them."""
    peak, median = _rates(metric, row)
    compiled = row.get("compiled") or {}
    audit = {key: compiled[key] for key in _DETAIL_KEYS if key in compiled}
    audit.update((key, row[key]) for key in _DETAIL_KEYS if key in row)
    return {"value": peak, "median_value": median,
            "smoke_only": bool(row.get("smoke_only", False)), **audit,
            "configuration": {key: row[key] for key in _CONFIG_KEYS if key in row}}


# Why a measured rate is kept but marked unverified: per group, the first rule
# whose test holds gives the reason; no rule holding means verified.
def _tensor_unit_unknown(metric: Metric, d: dict) -> bool:
    execution = d.get("execution_kind")
    unit_known = execution == "simt" or (execution == "tensor"
                                         and d.get("native_tensor_verified") is True)
    return d.get("instruction_precision_verified") is not True or not unit_known


def _vector_unverified(metric: Metric, d: dict) -> bool:
    return d.get("native_arithmetic_verified") is not True


_UNVERIFIED_RULES = {
    "Tensor": (
        (_tensor_unit_unknown,
         "Measured matrix rate retained; native instruction precision or execution unit is "
         "unverified"),
    ),
    "Vector": (
        (lambda m, d: (_vector_unverified(m, d) and m.precision == "int8"
                       and bool(d.get("includes_unpacking"))),
         "Measured portable INT8-input path uses INT32 arithmetic and includes unpacking; "
         "native INT8 execution is unverified"),
        (_vector_unverified,
         "Measured vector rate retained; native arithmetic instruction precision is unverified"),
    ),
}


def _verification_reason(metric: Metric, details: dict) -> str | None:
    return next((reason for test, reason in _UNVERIFIED_RULES.get(metric.group, ())
                 if test(metric, details)), None)


# summarize() is a chain of stages; each returns the finished row or None to
# hand the document on.  `view` carries what earlier stages derived.
_DECLARED_STATUSES = ("unsupported", "not_implemented", "error", "unavailable")


def _stage_declared(metric, document, view):
    status = document.get("status")
    if status in _DECLARED_STATUSES:
        return {**empty_metric(metric), "status": status,
                "reason": document.get("reason", status)}
    return None


def _stage_capacity(metric, document, view):
    if metric.key != "memory_capacity":
        return None
    capacity = document.get("device", {}).get("total_memory_bytes")
    if not _is_rate(capacity):
        return {**empty_metric(metric), "status": "unavailable",
                "reason": "Backend did not report total memory capacity"}
    return {**empty_metric(metric), "status": "ok", "value": capacity / 2**30,
            "capacity_bytes": capacity, "measurement_kind": "reported_device_capacity"}


def _stage_rows(metric, document, view):
    rows = document.get("results", [])
    if not isinstance(rows, list):
        return empty_metric(metric, "error", "Benchmark results must be a list")
    view["rows"] = [row for row in rows if isinstance(row, dict)]
    view["valid"] = [row for row in rows if _has_rates(metric, row)]
    if view["valid"]:
        return None
    rejected = view["rows"]
    reasons = "; ".join(dict.fromkeys(str(row.get("reason", "No valid throughput"))
                                      for row in rejected))
    all_unsupported = bool(rejected) and all(row.get("status") == "unsupported"
                                             for row in rejected)
    return empty_metric(metric, "unsupported" if all_unsupported else "error",
                        reasons or "Benchmark produced no valid throughput measurements")


def _hbm_sized(row) -> bool:
    return row.get("peak_eligible") is True and not row.get("smoke_only", False)


def _stage_bandwidth(metric, document, view):
    """Copy and read patterns are kept as details; only an HBM-sized copy row
    may give the metric's value."""
    if metric.key != "memory_bandwidth":
        return None
    patterns = {}
    for pattern in ("copy", "read"):
        rows = [row for row in view["valid"] if row.get("pattern") == pattern]
        pool = [row for row in rows if _hbm_sized(row)] or rows
        if pool:
            patterns[pattern] = _row_details(metric, max(pool, key=_peak_of(metric)))
    view["patterns"] = patterns
    view["valid"] = [row for row in view["valid"]
                     if row.get("pattern") == "copy" and _hbm_sized(row)]
    if view["valid"]:
        return None
    return {**empty_metric(metric), "patterns": patterns, "status": "not_measured",
            "reason": "No HBM-sized copy candidate: use a non-quick run with known L2 capacity "
                      "and buffers at least 4x L2; observed pattern rates remain in patterns"}


def _stage_best(metric, document, view):
    valid = view["valid"]
    result = {**empty_metric(metric), **({"patterns": view["patterns"]}
                                         if "patterns" in view else {}),
              "status": "ok", **_row_details(metric, max(valid, key=_peak_of(metric)))}
    if document.get("arguments", {}).get("quick") and metric.group != "Memory":
        result["smoke_only"] = True
    reason = _verification_reason(metric, result)
    if reason:
        result.update(status="unverified", reason=reason)
    result["successful_configurations"] = len(valid)
    return result


_SUMMARY_STAGES = (_stage_declared, _stage_capacity, _stage_rows, _stage_bandwidth, _stage_best)


def summarize(metric: Metric, document: dict) -> dict:
    """One table row from a child's declared status and validated measurement rows."""
    view: dict = {}
    for stage in _SUMMARY_STAGES:
        result = stage(metric, document, view)
        if result is not None:
            return result
    raise AssertionError("the last summary stage always returns a row")


_RUN_KEYS = ("command", "source_json", "log_file", "returncode", "device_index", "window",
             "patterns", "capacity_bytes", "partial_measurement", "reason", "value",
             "median_value", "status", "successful_configurations")


def aggregate_gpus(metric: Metric, rows: list[dict]) -> dict:
    """One table row for a metric measured concurrently on several GPUs.

    Each GPU runs its own independent probe (no collective), so the aggregate
    rate is the sum of the per-GPU peaks (medians) and the capacity the sum of
    the per-GPU capacities.  The row keeps the single-GPU schema; the detail
    fields come from the first GPU and every GPU's own row is kept under
    ``per_gpu``.  A rate is aggregated only when every GPU measured one.
    """
    result = empty_metric(metric)
    measured = [row for row in rows if row.get("status") in ("ok", "unverified")]
    values = [row.get("value") for row in measured]
    medians = [row.get("median_value") for row in measured]
    if rows and len(measured) == len(rows) and all(_is_rate(v) for v in values):
        result.update({k: v for k, v in rows[0].items() if k not in _RUN_KEYS})
        result["value"] = sum(values)
        result["median_value"] = sum(medians) if all(_is_rate(v) for v in medians) else None
        unverified = [row for row in rows if row["status"] == "unverified"]
        result["status"] = "unverified" if unverified else "ok"
        if unverified:
            result["reason"] = unverified[0].get("reason")
        if metric.key == "memory_capacity":
            result["capacity_bytes"] = sum(row.get("capacity_bytes", 0) for row in rows)
    else:
        statuses = {row.get("status") for row in rows}
        if len(statuses) == 1 and statuses <= {"unsupported", "not_implemented",
                                               "not_measured", "unavailable"}:
            result.update(status=statuses.pop(), reason=rows[0].get("reason"))
        else:
            failed = [row for row in rows if row not in measured]
            result.update(status="error", reason="; ".join(
                f"GPU {row.get('device_index', i)}: {row.get('status')}"
                + (f" ({row['reason']})" if row.get("reason") else "")
                for i, row in enumerate(failed)) or "no GPU produced a rate")
            if measured and all(_is_rate(v) for v in values):
                result["partial_measurement"] = {"gpus": len(measured), "value": sum(values)}
    per_gpu_values = [v for v in values if _is_rate(v)]
    result["aggregation"] = {
        "n_gpus": len(rows),
        "method": ("sum over GPUs of each GPU's value from concurrent, independent runs "
                   "(no collective)"),
        "per_gpu_value_min": min(per_gpu_values, default=None),
        "per_gpu_value_max": max(per_gpu_values, default=None),
    }
    result["per_gpu"] = rows
    return result


def format_per_gpu(results: list[dict]) -> str:
    """Metric x GPU table of the per-GPU values (empty when no row has per-GPU data)."""
    rows = [item for item in results if item.get("per_gpu")]
    if not rows:
        return ""
    devices = [sub.get("device_index", i) for i, sub in enumerate(rows[0]["per_gpu"])]
    header = f"{'Metric':<20} " + " ".join(f"{'GPU ' + str(d):>11}" for d in devices)
    lines = [header, "-" * len(header)]
    for item in rows:
        cells = []
        for sub in item["per_gpu"]:
            value = sub.get("value")
            cells.append(f"{value:>11.3f}" if _is_rate(value) else f"{sub.get('status', '-'):>11}")
        lines.append(f"{item['metric']:<20} " + " ".join(cells))
    return "\n".join(lines)


# The table: (header, width/alignment, cell) per column; the last column is
# unpadded.  Notes follow the table, one per matching (test, text) rule.
_TABLE_COLUMNS = (
    ("Metric", "<20", lambda item: item["metric"]),
    ("Peak / capacity", ">17",
     lambda item: "-" if item.get("value") is None else f"{item['value']:.3f}"),
    ("Median", ">12",
     lambda item: "-" if item.get("median_value") is None else f"{item['median_value']:.3f}"),
    ("Unit", "<8", lambda item: item["unit"]),
    ("Status", "", lambda item: item["status"]),
)
_TABLE_RULE_WIDTH = 86
_TABLE_NOTES = (
    (lambda item: item.get("reason"), lambda item: item["reason"]),
    (lambda item: item.get("smoke_only"), lambda item: "smoke test; not a peak result"),
    (lambda item: item.get("execution_kind") == "simt",
     lambda item: "measured matrix rate using SIMT scalar/vector instructions (no native "
                  "tensor MMA)"),
)


def format_table(results: list[dict]) -> str:
    """One line per requested metric, including missing results, then notes."""
    def line(cells):
        return " ".join(f"{cell:{spec}}" for cell, (_, spec, _) in zip(cells, _TABLE_COLUMNS))

    lines = [line([header for header, _, _ in _TABLE_COLUMNS]), "-" * _TABLE_RULE_WIDTH]
    lines += [line([cell(item) for _, _, cell in _TABLE_COLUMNS]) for item in results]
    notes = [f"{item['metric']}: {text(item)}" for item in results
             for test, text in _TABLE_NOTES if test(item)]
    return "\n".join(lines + (["", *notes] if notes else []))
