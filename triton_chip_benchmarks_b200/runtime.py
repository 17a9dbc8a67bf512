"""Device setup, device-event timing and result documents for the probes.

This is the runtime layer under the three probe drivers:

* :func:`setup_device` selects the CUDA device and records its metadata (the
  ``device`` block of every result document), from ``tcb_device_query``.
* :func:`measure` times a zero-argument launch function with device events
  around batches of launches captured in a CUDA graph (or plain event batches),
  following the reference suite's timing policy (common.py:306-534): the
  batch size is calibrated until the event timer resolves it, then refined
  towards ``--batch-ms``; after ``--warmup`` ms of replays at least ``--rounds``
  batches (and ``--rep`` ms) are sampled; a zero or too-coarse sample restarts
  the sampling with a larger batch.  Per-launch time = batch time / launches.
  Peak uses the minimum sample, sustained the median.
* :func:`emit_results`, :func:`emit_unsupported`, :func:`emit_not_implemented`
  write the child JSON document the suite summarizes (common.py:537-601).

The device API is duck-typed (``Event``, ``synchronize``, ``graph``,
``CUDAGraph``, ``Stream``, ``stream``); by default it is ``torch.cuda``.
Tests substitute a fake device with a deterministic clock.
"""

from __future__ import annotations

import argparse
from contextlib import nullcontext
from datetime import datetime, timezone
import json
import math
from pathlib import Path
import statistics

INITIAL_CALIBRATION_LAUNCHES = 5
MAX_BATCH_LAUNCHES = 2048
MIN_RESOLVED_EVENT_TICKS = 20

VENDOR = "nvidia"
DEVICE_TYPE = "cuda"


# ----------------------------------------------------------------- arguments
def positive_int(value):
    number = int(value)
    if number <= 0:
        raise argparse.ArgumentTypeError("must be a positive integer")
    return number


def positive_float(value):
    number = float(value)
    if not math.isfinite(number) or number <= 0:
        raise argparse.ArgumentTypeError("must be a finite positive number")
    return number


def add_common_arguments(parser: argparse.ArgumentParser) -> None:
    """The flags every probe accepts (reference common.py:117-133)."""
    parser.add_argument("--device", type=int, default=0, help="CUDA device index (default: 0)")
    parser.add_argument("--warmup", type=positive_float, default=100,
                        help="Approximate device warmup duration in ms (default: 100)")
    parser.add_argument("--rep", type=positive_float, default=200,
                        help="Approximate measurement budget in ms (default: 200)")
    parser.add_argument("--timing", choices=("auto", "graph", "events"), default="auto",
                        help="auto uses CUDA graph batches, falling back to event batches")
    parser.add_argument("--batch-ms", type=positive_float, default=10,
                        help="Target batch duration in ms (default: 10)")
    parser.add_argument("--rounds", type=positive_int, default=10,
                        help="Minimum number of measured batches (default: 10)")
    parser.add_argument("--compute-units", type=positive_int,
                        help="Override the SM count reported by the device")
    parser.add_argument("--l2-mib", type=positive_float,
                        help="Override the L2 capacity in MiB reported by the device")
    parser.add_argument("--output", type=Path, help="Save metadata and all samples as JSON")


# -------------------------------------------------------------------- device
def setup_device(args, *, announce: bool = True) -> dict:
    """Select ``args.device`` and describe it (reference common.py:214-292)."""
    import torch

    from . import _native

    if not torch.cuda.is_available():
        raise SystemExit("No CUDA device is available")
    count = torch.cuda.device_count()
    if not 0 <= args.device < count:
        raise SystemExit(f"Invalid --device {args.device}; available indices: 0..{count - 1}")
    torch.cuda.set_device(args.device)
    torch.manual_seed(0)
    props = _native.device_query(args.device)
    units, unit_source = props.sm_count, "cudaDeviceProp.multiProcessorCount"
    if getattr(args, "compute_units", None) is not None:
        units, unit_source = args.compute_units, "--compute-units"
    l2, l2_source = int(props.l2_cache_bytes), "cudaDeviceProp.l2CacheSize"
    if getattr(args, "l2_mib", None) is not None:
        l2, l2_source = int(args.l2_mib * 2**20), "--l2-mib"
    total = int(props.total_mem_bytes)
    metadata = {
        "device_index": args.device, "device_type": DEVICE_TYPE,
        "device_name": props.name, "vendor_name": VENDOR,
        "backend": "cuda", "architecture": f"sm_{props.major}{props.minor}a",
        "compute_capability": f"{props.major}.{props.minor}",
        "sm_count": units, "compute_units_source": unit_source,
        "total_memory_bytes": total, "memory_capacity_gib": total / 2**30,
        "l2_cache_bytes": l2, "l2_cache_source": l2_source,
        "max_shared_memory_per_block": props.max_smem_per_block,
        "sm_clock_max_mhz": props.clock_khz / 1000.0,
        "memory_clock_max_mhz": props.mem_clock_khz / 1000.0,
        "memory_bus_width_bits": props.mem_bus_width,
        "supports_fp64": True, "supports_bf16": True,
        "torch_version": torch.__version__,
        "tcb_version": _native.version(),
        "cuda_driver_version": props.driver_version,
        "cuda_runtime_version": props.runtime_version,
        "device_api": "torch.cuda",
    }
    if announce:
        print(f"Device cuda:{args.device}: {props.name} | sm_{props.major}{props.minor} | "
              f"SMs={units} | memory={total / 2**30:.1f} GiB | L2={l2 / 2**20:.0f} MiB")
        print(f"libtcb {metadata['tcb_version']}, PyTorch {torch.__version__}; "
              f"timing={args.timing}, warmup={args.warmup:g} ms, rep={args.rep:g} ms")
    return metadata


def available_memory_bytes() -> int | None:
    import torch
    try:
        return int(torch.cuda.mem_get_info()[0])
    except RuntimeError:
        return None


# -------------------------------------------------------------------- timing
def _quantile(samples, q):
    ordered = sorted(samples)
    pos = (len(ordered) - 1) * q
    lo, hi = math.floor(pos), math.ceil(pos)
    return ordered[lo] + (ordered[hi] - ordered[lo]) * (pos - lo)


class GraphUnavailable(RuntimeError):
    """The device API offers no usable graph capture."""


def _default_api():
    import torch
    return torch.cuda


def _graph_class(api):
    if not all(callable(getattr(api, name, None)) for name in ("graph", "Stream", "stream")):
        return None, None
    for name in ("CUDAGraph", "Graph"):
        factory = getattr(api, name, None)
        if callable(factory):
            return factory, name
    return None, None


def _timed_stream(api):
    if callable(getattr(api, "Stream", None)) and callable(getattr(api, "stream", None)):
        return api.stream(api.Stream())
    return nullcontext()


def _zero_time_error(launches=None):
    scope = f" for {launches} launches" if launches is not None else ""
    return RuntimeError(f"Invalid device event time: 0 ms{scope}; the event timer is "
                        "unavailable or too coarse for this workload")


def _coarse_time_error(launches, elapsed_ms, needed_ms):
    return RuntimeError(f"Device event resolution too coarse: {launches} launches measured "
                        f"{elapsed_ms:g} ms, but at least {needed_ms:g} ms is needed")


def _grow(launches):
    return min(MAX_BATCH_LAUNCHES, launches * 2)


class _BatchTimer:
    """The batch-timing policy as a small phase machine.

    Each phase is a method that does its device work and returns the name of
    the next phase:

    calibrate  direct batches of 5, 10, 20 ... launches until the event timer
               reads a nonzero time; that gives the per-launch estimate and,
               when a zero reading came first, a floor of 20 readings' worth
               of time that every later batch must reach;
    size       the batch that fills min(--batch-ms, --rep / --rounds), built
               (one captured graph in graph mode) and made resolvable;
    refine     up to two re-sizings toward that target, skipped once the
               batch time lies within a factor of two of it;
    warm       replays of the batch for --warmup ms;
    recapture  the batch built and resolved once more after warm-up;
    sample     max(--rounds, --rep / batch time) resolved batch times.  An
               unresolved sample doubles the batch, rebuilds it and returns
               to ``sample``, which starts over, so all samples share one
               launch count.

    A batch is "resolved" when it reads a nonzero time at or above the floor;
    building doubles the launch count (up to MAX_BATCH_LAUNCHES) until it is.
    """

    REFINE_PASSES = 2

    def __init__(self, fn, api, graph_class, args):
        self.fn, self.api, self.graph_class, self.args = fn, api, graph_class, args
        self.start = api.Event(enable_timing=True)
        self.end = api.Event(enable_timing=True)
        self.target_ms = min(args.batch_ms, args.rep / args.rounds)
        self.floor_ms = 0.0
        self.per_launch_ms = 0.0
        self.calibration_launches = 0
        self.min_launches = 1
        self.refines_left = self.REFINE_PASSES
        self.launches, self.submit, self.batch_ms = 0, None, 0.0
        self.samples: list[float] = []

    # ---------------------------------------------------------- device work
    def _run_direct(self, count):
        for _ in range(count):
            self.fn()

    def _read(self, submit) -> float:
        """Device time of one submission (zero allowed: a coarse timer's reading)."""
        self.start.record()
        submit()
        self.end.record()
        self.api.synchronize()
        ms = float(self.start.elapsed_time(self.end))
        if not math.isfinite(ms) or ms < 0:
            raise RuntimeError(f"Invalid device event time: {ms!r} ms")
        return ms

    def _build(self, count):
        """A submission of `count` launches: a captured graph's replay, or direct."""
        if self.graph_class is None:
            return lambda: self._run_direct(count)
        try:
            graph = self.graph_class()
            with self.api.graph(graph):
                self._run_direct(count)
        except NotImplementedError as exc:
            raise GraphUnavailable(f"graph capture: {exc}") from exc
        except RuntimeError as exc:
            text = str(exc).lower()
            if any(w in text for w in ("not supported", "unsupported", "not implemented")):
                raise GraphUnavailable(f"graph capture: {exc}") from exc
            raise
        return graph.replay

    def _resolved(self, ms: float) -> bool:
        return ms > 0 and ms >= self.floor_ms

    def _unresolvable(self, count, ms):
        error = (_zero_time_error(count) if ms == 0
                 else _coarse_time_error(count, ms, self.floor_ms))
        return GraphUnavailable(f"graph timing: {error}") if self.graph_class else error

    def _clamp(self, count: int) -> int:
        return max(self.min_launches, min(MAX_BATCH_LAUNCHES, count))

    def _resolve(self, count: int, zero_seen: bool = False) -> None:
        """Build batches from `count` launches up, doubling, until one resolves."""
        while True:
            submit = self._build(count)
            ms = self._read(submit)
            if ms > 0 and zero_seen and self.floor_ms == 0:
                self.floor_ms = ms * MIN_RESOLVED_EVENT_TICKS
            if self._resolved(ms):
                self.launches, self.submit, self.batch_ms = count, submit, ms
                return
            if count == MAX_BATCH_LAUNCHES:
                raise self._unresolvable(count, ms)
            zero_seen = zero_seen or ms == 0
            count = _grow(count)

    # --------------------------------------------------------------- phases
    def calibrate(self) -> str:
        launches, saw_zero = INITIAL_CALIBRATION_LAUNCHES, False
        while True:
            ms = self._read(lambda: self._run_direct(launches))
            if ms > 0:
                break
            if launches == MAX_BATCH_LAUNCHES:
                raise _zero_time_error(launches)
            saw_zero, launches = True, _grow(launches)
        self.per_launch_ms = max(ms / launches, 0.001)
        self.calibration_launches = launches
        if saw_zero:
            self.min_launches = launches
            self.floor_ms = ms * MIN_RESOLVED_EVENT_TICKS
        return "size"

    def size(self) -> str:
        self._resolve(self._clamp(math.ceil(self.target_ms / self.per_launch_ms)))
        return "refine"

    def refine(self) -> str:
        if self.refines_left == 0 or 0.5 * self.target_ms <= self.batch_ms <= 2 * self.target_ms:
            return "warm"
        resized = self._clamp(math.ceil(self.launches * self.target_ms / self.batch_ms))
        if resized == self.launches:
            return "warm"
        self.refines_left -= 1
        self._resolve(resized)
        return "refine"

    def warm(self) -> str:
        for _ in range(max(1, math.ceil(self.args.warmup / self.batch_ms))):
            self.submit()
        self.api.synchronize()
        return "recapture"

    def recapture(self) -> str:
        self._resolve(self.launches)
        return "sample"

    def sample(self) -> str:
        wanted = max(self.args.rounds, math.ceil(self.args.rep / self.batch_ms))
        self.samples = []
        while len(self.samples) < wanted:
            ms = self._read(self.submit)
            if self._resolved(ms):
                self.samples.append(ms)
                continue
            if self.launches == MAX_BATCH_LAUNCHES:
                raise self._unresolvable(self.launches, ms)
            self._resolve(_grow(self.launches), zero_seen=ms == 0)
            return "sample"
        return "done"

    def run(self) -> list[float]:
        phase = "calibrate"
        while phase != "done":
            phase = getattr(self, phase)()
        return self.samples


def _batch_samples(fn, args, api, use_graph):
    """Per-launch times (batch time / launches) and the batch details."""
    graph_class, graph_name = _graph_class(api) if use_graph else (None, None)
    if use_graph and graph_class is None:
        raise GraphUnavailable("the device API exposes no graph capture")
    with _timed_stream(api):
        timer = _BatchTimer(fn, api, graph_class, args)
        batches = timer.run()
    return [ms / timer.launches for ms in batches], {
        "launches_per_batch": timer.launches, "batch_samples_ms": batches,
        "sample_count": len(batches), "measured_total_ms": sum(batches),
        "graph_api": graph_name, "calibration_launches": timer.calibration_launches,
        "minimum_resolved_batch_ms": timer.floor_ms,
    }


def measure(fn, args, api=None) -> dict:
    """Device-event timing of ``fn`` (never a host wall clock).

    With the default CUDA device API the SM clock and throttle reasons are
    sampled during the timed batches and returned under ``clocks``.
    """
    if api is None:
        from .clocks import ClockSampler
        import torch
        with ClockSampler(torch.cuda.current_device()) as sampler:
            result = _measure(fn, args, _default_api())
        result["clocks"] = sampler.summary()
        return result
    return _measure(fn, args, api)


def _measure(fn, args, api) -> dict:
    if not all(callable(getattr(api, name, None)) for name in ("Event", "synchronize")):
        raise RuntimeError("The device API does not expose timed events")
    fn()  # first launch outside any capture and any sample
    api.synchronize()
    requested = args.timing
    # Graph batches first unless plain events were asked for; "auto" falls back
    # to event batches when graph capture or graph timing is unavailable.
    modes = {"events": ("events",), "graph": ("graph",), "auto": ("graph", "events")}[requested]
    fallback = None
    for selected in modes:
        try:
            samples, details = _batch_samples(fn, args, api, use_graph=selected == "graph")
            break
        except (GraphUnavailable, NotImplementedError) as exc:
            if selected == modes[-1]:
                raise
            api.synchronize()
            fallback = str(exc)
    if not samples or any(not math.isfinite(v) or v <= 0 for v in samples):
        raise RuntimeError("Invalid device timing; increase the workload or --rep")
    notice = f"Timing: {selected} via device events"
    if fallback:
        notice += f" (auto fallback: {fallback}; includes host dispatch gaps)"
    if getattr(args, "_timing_notice", None) != notice:
        print(notice)
        args._timing_notice = notice
    return {
        "median_ms": statistics.median(samples), "p20_ms": _quantile(samples, 0.2),
        "p80_ms": _quantile(samples, 0.8), "min_ms": min(samples), "max_ms": max(samples),
        "timing_method": selected, "timing_requested": requested,
        "timing_fallback_reason": fallback, "samples_ms_per_launch": samples, **details,
    }


# ------------------------------------------------------------------- results
def _serialized_arguments(args) -> dict:
    return {key: str(value) if isinstance(value, Path) else value
            for key, value in vars(args).items() if not key.startswith("_")}


def write_document(args, document) -> None:
    if getattr(args, "output", None) is None:
        return
    args.output.parent.mkdir(parents=True, exist_ok=True)
    args.output.write_text(json.dumps(document, indent=2, ensure_ascii=False,
                                      allow_nan=False) + "\n")
    print(f"JSON: {args.output.resolve()}")


def _now() -> str:
    return datetime.now(timezone.utc).isoformat()


def _emit_no_measurement(name, metadata, args, reason, status, *, details=None):
    document = {"benchmark": name, "status": status, "reason": str(reason),
                "timestamp_utc": _now(), "device": metadata,
                "arguments": _serialized_arguments(args), "results": []}
    if details is not None:
        document["details"] = details
    print(f"{status.upper()}: {reason}")
    write_document(args, document)
    return document


def emit_unsupported(name, metadata, args, reason, *, details=None):
    """An explicit device or library capability rejection."""
    return _emit_no_measurement(name, metadata, args, reason, "unsupported", details=details)


def emit_not_implemented(name, metadata, args, reason, *, details=None):
    """A gap in this benchmark, not a claim about the device."""
    return _emit_no_measurement(name, metadata, args, reason, "not_implemented", details=details)


def emit_results(name, metadata, args, rows):
    if not rows:
        raise RuntimeError("No valid measurements were produced")
    methods = sorted({row["timing_method"] for row in rows if "timing_method" in row})
    document = {
        "benchmark": name, "status": "ok", "timestamp_utc": _now(), "device": metadata,
        "arguments": _serialized_arguments(args),
        "timing": {
            "provider": "torch.cuda.Event (CUDA events) around CUDA-graph batches",
            "requested": args.timing, "methods_used": methods,
            "method": "device events around batches; elapsed / actual launch count; no cache flush",
            "peak_statistic": "minimum sampled batch-average device time",
            "sustained_statistic": "median sampled batch-average device time",
            "includes": "kernel work, device scheduling and amortized event overhead; "
                        "events mode additionally includes host dispatch gaps",
            "excludes": "library load, allocation, initialization, validation, capture and warmup",
        },
        "results": rows,
    }
    write_document(args, document)
    return document
