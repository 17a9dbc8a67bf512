#!/usr/bin/env python3
"""Run the complete 17-row chip metric table on B200s, one child per metric.

Drop-in for the reference suite runner (bench_suite.py:50-203): the same
flags, one isolated child process per metric with a timeout, stale output
removed before each child, the combined report rewritten atomically after
every metric, and a final table.  Children are this package's probe drivers
(bench_bandwidth, bench_tensor, bench_vector) running libtcb kernels.

With --gpus N each metric's child runs concurrently on GPUs DEVICE ..
DEVICE+N-1 (the probes are independent per device: no collective, no
NCCL).  Every GPU's document is summarized into a per-GPU sub-row and the
table row carries the aggregate (sum of per-GPU peaks and medians), in the
same chip_metric_suite schema.
"""

from __future__ import annotations

import argparse
from datetime import datetime, timezone
import json
from pathlib import Path
import subprocess
import sys
import time

from .runtime import positive_float, positive_int
from .suite_report import (METRICS, aggregate_gpus, empty_metric, format_per_gpu, format_table,
                           summarize)

REPO_ROOT = Path(__file__).resolve().parent.parent
PACKAGE = __package__ or "triton_chip_benchmarks_b200"

MEASUREMENT_POLICY = (
    "Highest observed valid throughput; median from the same configuration. Capacity is "
    "reported device capacity. Bandwidth is effective copy read+write traffic with HBM-sized "
    "buffers; read rates are auxiliary details. Unsupported and not-implemented metrics have no "
    "numeric value; errors do not imply unsupported hardware.")


def build_parser():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--device", type=int, default=0)
    parser.add_argument("--gpus", type=positive_int, default=1,
                        help="run every metric concurrently on GPUs DEVICE..DEVICE+N-1 and "
                             "report the aggregate with per-GPU sub-rows (default: 1)")
    parser.add_argument("--timing", choices=("auto", "graph", "events"), default="auto")
    parser.add_argument("--warmup", type=positive_float, default=100)
    parser.add_argument("--rep", type=positive_float, default=200)
    parser.add_argument("--batch-ms", type=positive_float, default=10)
    parser.add_argument("--rounds", type=positive_int, default=10)
    parser.add_argument("--compute-units", type=positive_int)
    parser.add_argument("--l2-mib", type=positive_float)
    parser.add_argument("--quick", action="store_true",
                        help="Smoke checks; these rates are not peak measurements")
    parser.add_argument("--output", type=Path, default=Path("results/chip_metrics.json"),
                        help="Complete table JSON, checkpointed after every metric")
    parser.add_argument("--results-dir", type=Path,
                        help="Per-metric raw JSON and logs (default: OUTPUT_STEM_runs)")
    parser.add_argument("--timeout", type=positive_float, default=900,
                        help="Maximum seconds per metric (default: 900)")
    parser.add_argument("--metrics", nargs="+", help="Run only these metric keys")
    parser.add_argument("--probe-device", action="store_true", help=argparse.SUPPRESS)
    return parser


def metric_command(metric, args, output: Path, device: int | None = None) -> list[str]:
    """The child command for one metric on one device (no shell)."""
    device = args.device if device is None else device
    if metric.key == "memory_capacity":
        module, extra = "bench_suite", ["--probe-device"]
    elif metric.key == "memory_bandwidth":
        module, extra = "bench_bandwidth", ["--mode", "all", "--dtype", "fp32"]
    elif metric.group == "Tensor":
        module = "bench_tensor"
        extra = ["--mode", "peak", "--dtype",
                 "fp32" if metric.precision == "tf32" else metric.precision]
        if metric.precision in ("fp32", "tf32"):
            extra += ["--input-precision", "tf32" if metric.precision == "tf32" else "ieee"]
    else:
        module, extra = "bench_vector", ["--dtype", metric.precision]
    command = [sys.executable, "-u", "-m", f"{PACKAGE}.{module}", *extra,
               "--device", str(device), "--timing", args.timing,
               "--warmup", str(args.warmup), "--rep", str(args.rep),
               "--batch-ms", str(args.batch_ms), "--rounds", str(args.rounds),
               "--output", str(output)]
    for flag, value in (("--compute-units", args.compute_units), ("--l2-mib", args.l2_mib)):
        if value is not None:
            command += [flag, str(value)]
    if args.quick:
        command.append("--quick")
    return command


def write_json(path: Path, document: dict) -> None:
    """Atomic replace, so a reader never sees a half-written report."""
    path.parent.mkdir(parents=True, exist_ok=True)
    temporary = path.with_name(path.name + ".tmp")
    temporary.write_text(json.dumps(document, indent=2, allow_nan=False) + "\n")
    temporary.replace(path)


def probe_device(args) -> None:
    from .runtime import setup_device
    metadata = setup_device(args)
    write_json(args.output, {"status": "ok", "device": metadata, "results": []})


# Statuses a child declares about the device or the benchmark (its exit code
# does not turn them into errors), and statuses that carry a measured rate.
_DECLARED_GAPS = ("unsupported", "not_implemented")
_MEASURED = ("ok", "unverified")


def _child_document(output: Path):
    """(document, None) from the child's JSON, or (None, why it is unusable)."""
    if not output.exists():
        return None, "Benchmark did not write result JSON"
    try:
        document = json.loads(output.read_text())
    except (OSError, ValueError) as exc:
        return None, f"Invalid benchmark JSON: {exc}"
    if not isinstance(document, dict):
        return None, "Invalid benchmark JSON: expected a JSON object"
    return document, None


def _summarized(metric, args, document: dict) -> dict:
    try:
        row = summarize(metric, document)
    except (ValueError, TypeError, AttributeError, KeyError) as exc:
        return empty_metric(metric, "error", f"Invalid benchmark JSON: {exc}")
    if args.quick and row["status"] in _MEASURED and metric.group != "Memory":
        row["smoke_only"] = True
    return row


def conclude(metric, args, output: Path, returncode, failure: str | None = None):
    """Table row from a finished child: its JSON, exit code, or the failure text.

    A child that could not run (`failure`) or left no usable JSON is an error.
    A non-zero exit is an error whatever the child wrote, unless it declared a
    capability gap; a rate it did write is kept as ``partial_measurement``.
    """
    if failure is not None:
        return empty_metric(metric, "error", failure), None
    document, problem = _child_document(output)
    row = (empty_metric(metric, "error", problem) if document is None
           else _summarized(metric, args, document))
    if returncode and row["status"] not in _DECLARED_GAPS:
        failed = empty_metric(metric, "error", f"Benchmark exited with code {returncode}; see log")
        if row["status"] in _MEASURED:
            failed["partial_measurement"] = row
        row = failed
    return row, document


def run_metric(metric, args, directory: Path, runner=subprocess.run):
    output = directory / f"{metric.key}.json"
    log = directory / f"{metric.key}.log"
    command = metric_command(metric, args, output)
    output.unlink(missing_ok=True)  # a stale success must never stand in for a failed run
    returncode = failure = None
    try:
        with log.open("w") as stream:
            completed = runner(command, cwd=REPO_ROOT, stdout=stream, stderr=subprocess.STDOUT,
                               timeout=args.timeout, check=False)
        returncode = completed.returncode
    except subprocess.TimeoutExpired:
        failure = f"Exceeded {args.timeout:g} seconds; see log"
    except OSError as exc:
        failure = f"Cannot execute benchmark: {exc}"
    result, document = conclude(metric, args, output, returncode, failure)
    result.update(command=command, source_json=str(output), log_file=str(log),
                  returncode=returncode)
    return result, document


def window_overlap(windows) -> float | None:
    """Time all child windows share, over the shortest window (1.0 = fully concurrent)."""
    if not windows:
        return None
    common = min(end for _, end in windows) - max(start for start, _ in windows)
    shortest = min(end - start for start, end in windows)
    return max(0.0, common) / shortest if shortest > 0 else 1.0


def run_metric_gpus(metric, args, directory: Path, popen=subprocess.Popen, clock=time.time):
    """One metric on args.gpus devices at once; the row is the per-GPU aggregate."""
    devices = [args.device + i for i in range(args.gpus)]
    launched = []
    for device in devices:
        output = directory / f"{metric.key}.gpu{device}.json"
        log = directory / f"{metric.key}.gpu{device}.log"
        output.unlink(missing_ok=True)
        command = metric_command(metric, args, output, device)
        stream = log.open("w")
        proc = failure = None
        try:
            proc = popen(command, cwd=REPO_ROOT, stdout=stream, stderr=subprocess.STDOUT)
        except OSError as exc:
            failure = f"Cannot execute benchmark: {exc}"
        launched.append((device, output, log, command, stream, proc, clock(), failure))
    deadline = clock() + args.timeout
    rows, documents, windows = [], [], []
    for device, output, log, command, stream, proc, start, failure in launched:
        returncode = None
        if proc is not None:
            try:
                returncode = proc.wait(timeout=max(0.0, deadline - clock()))
            except subprocess.TimeoutExpired:
                proc.kill()
                proc.wait()
                failure = f"Exceeded {args.timeout:g} seconds; see log"
        stream.close()
        end = clock()
        result, document = conclude(metric, args, output, returncode, failure)
        result.update(device_index=device, window=[start, end], command=command,
                      source_json=str(output), log_file=str(log), returncode=returncode)
        rows.append(result)
        documents.append(document)
        if proc is not None and failure is None:
            windows.append((start, end))
    aggregate = aggregate_gpus(metric, rows)
    aggregate["aggregation"]["concurrent_window_overlap"] = window_overlap(windows)
    return aggregate, documents


def run_suite(args, runner=subprocess.run, popen=subprocess.Popen) -> dict:
    args.output = args.output.resolve()
    directory = (args.results_dir or args.output.with_name(args.output.stem + "_runs")).resolve()
    directory.mkdir(parents=True, exist_ok=True)
    selected = [m for m in METRICS if not args.metrics or m.key in args.metrics]
    gpus = getattr(args, "gpus", 1)
    report = {
        "schema_version": 1, "benchmark": "chip_metric_suite",
        "timestamp_utc": datetime.now(timezone.utc).isoformat(),
        "status": "running", "device": {}, "smoke_only": args.quick,
        "measurement_policy": MEASUREMENT_POLICY,
        "results": [empty_metric(m) for m in selected],
    }
    if gpus > 1:
        report["n_gpus"] = gpus
        report["devices"] = [None] * gpus
        report["multi_gpu_policy"] = (
            "Each metric runs concurrently and independently on every GPU (no collective); "
            "the row value is the sum of the per-GPU values, per-GPU rows under per_gpu.")
    write_json(args.output, report)
    for index, metric in enumerate(selected):
        print(f"[{index + 1}/{len(selected)}] {metric.key} ...", flush=True)
        if gpus > 1:
            result, documents = run_metric_gpus(metric, args, directory, popen)
            for slot, document in enumerate(documents):
                if document and document.get("device") and report["devices"][slot] is None:
                    report["devices"][slot] = document["device"]
            document = next((d for d in documents if d), None)
        else:
            result, document = run_metric(metric, args, directory, runner)
        report["results"][index] = result
        if document and document.get("device") and not report["device"]:
            report["device"] = document["device"]
        write_json(args.output, report)
        print(f"  {result['status']}" + (f": {result['reason']}" if result.get("reason") else ""),
              flush=True)
    report["status"] = "complete_with_errors" if any(
        item["status"] == "error" for item in report["results"]) else "complete"
    write_json(args.output, report)
    print("\n" + format_table(report["results"]))
    per_gpu = format_per_gpu(report["results"])
    if per_gpu:
        print("\nPer GPU:\n" + per_gpu)
    print(f"\nJSON: {args.output}")
    print(f"Raw results and logs: {directory}")
    return report


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    if args.probe_device:
        probe_device(args)
        return 0
    report = run_suite(args)
    return 1 if report["status"] == "complete_with_errors" else 0


if __name__ == "__main__":
    raise SystemExit(main())
