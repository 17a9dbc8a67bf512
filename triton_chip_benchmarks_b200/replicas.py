#!/usr/bin/env python3
"""Run one probe configuration concurrently on N GPUs as independent replicas.

The probes have no exchange step, so N GPUs are N independent replicas: one
child process per GPU, each timing its own device with the suite's timing
policy.  A host barrier (a torch.distributed TCPStore on 127.0.0.1) aligns the
timed windows; each child posts its result to the store.  The parent reports
per-GPU peak/median, the aggregate (sum of per-GPU peaks), and marks the
aggregate valid only when every GPU spent at least 90 % of its timed window
concurrently with all the others.  A child
that fails or exceeds --timeout becomes an `error` entry for its GPU; the
others still report (the isolation rule of the suite runner, bench_suite.py:117-155).

  python -m triton_chip_benchmarks_b200.replicas --gpus 8 --probe tensor --dtype bf16 \
      --tile 256x256x64 --output results/replicas_bf16.json
"""

from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
import subprocess
import sys
import time

PACKAGE = __package__ or "triton_chip_benchmarks_b200"
OVERLAP_REQUIRED = 0.9


def build_parser():
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--probe", choices=("copy", "tensor", "vector", "fake"), required=True)
    parser.add_argument("--timeout", type=float, default=900.0,
                        help="seconds per child, including setup (default: 900)")
    parser.add_argument("--barrier-timeout", type=float, default=300.0)
    parser.add_argument("--output", type=Path)
    # probe configuration
    parser.add_argument("--mib", type=int, default=4096, help="copy: bytes per buffer in MiB")
    parser.add_argument("--variant", choices=("ldg128", "bulk"), default="ldg128")
    parser.add_argument("--dtype", default="bf16")
    parser.add_argument("--kernel", choices=("tcgen05", "dmma", "simt", "simt_reg"),
                        default="tcgen05")
    parser.add_argument("--tile", default="256x256x64")
    parser.add_argument("--chains", type=int, default=1)
    parser.add_argument("--blocks-per-sm", type=int, default=1)
    parser.add_argument("--iterations", type=int, default=4096)
    parser.add_argument("--threads", type=int, default=256)
    parser.add_argument("--elems", type=int, default=2)
    parser.add_argument("--unroll", type=int, default=8)
    parser.add_argument("--int8-op", default="dp4a")
    # timing policy (runtime.measure)
    parser.add_argument("--timing", choices=("auto", "graph", "events"), default="auto")
    parser.add_argument("--warmup", type=float, default=100.0)
    parser.add_argument("--rep", type=float, default=200.0)
    parser.add_argument("--batch-ms", type=float, default=10.0)
    parser.add_argument("--rounds", type=int, default=10)
    # child plumbing and CPU test hooks
    parser.add_argument("--child", action="store_true", help=argparse.SUPPRESS)
    parser.add_argument("--rank", type=int, default=0, help=argparse.SUPPRESS)
    parser.add_argument("--store-port", type=int, default=0, help=argparse.SUPPRESS)
    parser.add_argument("--fake-ms", type=float, default=1.0, help=argparse.SUPPRESS)
    parser.add_argument("--fake-fail-rank", type=int, default=-1, help=argparse.SUPPRESS)
    parser.add_argument("--fake-hang-rank", type=int, default=-1, help=argparse.SUPPRESS)
    return parser


# ----------------------------------------------------------------- probes
def prepare(args):
    """(run, operations, unit, config) for this child's device."""
    if args.probe == "fake":
        return prepare_fake(args)
    import torch

    from . import _native
    torch.cuda.set_device(args.rank)
    device = torch.device("cuda", args.rank)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    if args.probe == "copy":
        n = args.mib << 20
        src = torch.randint(0, 256, (n,), dtype=torch.uint8, device=device)
        dst = torch.zeros_like(src)
        variant = {"ldg128": _native.COPY_LDG128, "bulk": _native.COPY_BULK}[args.variant]

        def run():
            _native.copy(src, dst, n, variant, 0, 0)

        run()
        torch.cuda.synchronize()
        if not torch.equal(src, dst):
            raise AssertionError("copy validation failed")
        return run, 2 * n, "GB/s", {"bytes": n, "variant": args.variant}
    if args.probe == "tensor":
        from .bench_tensor import VARIANTS, launch, peak_inputs, reference_output
        from .validation import validate_relative
        m, n, k = (int(v) for v in args.tile.split("x"))
        variant = VARIANTS[args.kernel]
        config = dict(block_m=m, block_n=n, block_k=k, chains=args.chains, variant=variant)
        blocks = sms * args.blocks_per_sm
        gen = torch.Generator().manual_seed(args.rank)
        a, b, c, extras = peak_inputs(args.dtype, "baseline", blocks, config, device, gen)

        def run():
            launch(args.dtype, config, a, b, c, extras, blocks, args.blocks_per_sm,
                   args.iterations)

        run()
        torch.cuda.synchronize()
        validate_relative(c, reference_output(args.dtype, a, b, extras, args.iterations),
                          1e-3 if args.dtype in ("bf16", "fp16", "tf32") else
                          1e-12 if args.dtype == "fp64" else 1e-5 if args.dtype == "fp32"
                          else 0.0)
        ops = 2 * m * n * k * args.iterations * args.chains * blocks
        unit = "TOP/s" if args.dtype == "int8" else "TFLOP/s"
        return run, ops, unit, {"dtype": args.dtype, "kernel": args.kernel, "tile": args.tile,
                                "blocks": blocks, "iterations": args.iterations}
    from .bench_vector import make_inputs, native_dtype, validate
    ns = argparse.Namespace(dtype=args.dtype, int8_op=args.int8_op, inputs="baseline",
                            seed=args.rank)
    blocks = sms * args.blocks_per_sm
    elements = blocks * args.threads * args.elems
    x, coeff = make_inputs(ns, elements, device)
    out = torch.empty_like(x)
    code = native_dtype(ns)

    # Registers or by value per op; a host copy is made once, outside timing.
    coeff_arg = _native.vector_coefficients(code, coeff, coeff.cpu())

    def run():
        _native.vector_chains(code, x, out, coeff_arg, elements, args.iterations, blocks,
                              args.threads, args.elems, args.unroll)

    run()
    torch.cuda.synchronize()
    validate(ns, x, out, coeff, args.iterations)
    per_update = 8 if args.dtype == "int8" and args.int8_op == "dp4a" else 2
    unit = "TOP/s" if args.dtype == "int8" else "TFLOP/s"
    return run, per_update * 8 * elements * args.iterations, unit, {
        "dtype": args.dtype, "elements": elements, "iterations": args.iterations}


def prepare_fake(args):
    """A CPU stand-in with a deterministic device clock (tests only)."""
    if args.rank == args.fake_fail_rank:
        raise RuntimeError(f"planted failure on rank {args.rank}")
    if args.rank == args.fake_hang_rank:
        time.sleep(3600)
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "tests"))
    from fake_device import FakeDeviceAPI
    api = FakeDeviceAPI(kernel_ms=args.fake_ms * (1 + 0.01 * args.rank))

    def launch():
        api.launch()
        time.sleep(args.fake_ms / 1000.0)  # real time passes too, so host windows have length

    return launch, 10**9, "GB/s", {"fake_ms": args.fake_ms, "_api": api}


# ------------------------------------------------------------------ child
def child_main(args) -> int:
    from torch.distributed import TCPStore
    store = TCPStore("127.0.0.1", args.store_port, None, False,
                     timeout=__import__("datetime").timedelta(seconds=args.timeout))
    key = f"result/{args.rank}"
    try:
        run, operations, unit, config = prepare(args)
        api = config.pop("_api", None)
        store.add("ready", 1)
        deadline = time.time() + args.barrier_timeout
        barrier_ok = True
        while store.add("ready", 0) < args.gpus:
            if time.time() > deadline:
                barrier_ok = False
                break
            time.sleep(0.001)
        from .runtime import measure
        start = time.time()
        timing = measure(run, args, api=api) if api is not None else measure(run, args)
        end = time.time()
        if unit == "GB/s":
            peak = operations / (timing["min_ms"] * 1e6)
            median = operations / (timing["median_ms"] * 1e6)
        else:
            peak = operations / (timing["min_ms"] * 1e9)
            median = operations / (timing["median_ms"] * 1e9)
        result = {"rank": args.rank, "device": args.rank, "status": "ok", "unit": unit,
                  "peak": peak, "median": median, "operations": operations,
                  "window_start": start, "window_end": end, "barrier_ok": barrier_ok,
                  "config": config, "clocks": timing.get("clocks"),
                  "min_ms": timing["min_ms"], "median_ms": timing["median_ms"],
                  "timing_method": timing["timing_method"]}
    except Exception as exc:  # noqa: BLE001 - reported as this GPU's error
        store.add("ready", 1)
        result = {"rank": args.rank, "device": args.rank, "status": "error",
                  "reason": f"{type(exc).__name__}: {exc}"}
    store.set(key, json.dumps(result))
    return 0 if result["status"] == "ok" else 1


# ----------------------------------------------------------------- parent
def overlap_fraction(windows) -> float:
    """Time all windows share, over the shortest window (1.0 = fully concurrent)."""
    if not windows:
        return 0.0
    common = min(w[1] for w in windows) - max(w[0] for w in windows)
    shortest = min(w[1] - w[0] for w in windows)
    return max(0.0, common) / shortest if shortest > 0 else 1.0


def aggregate(results: list[dict], n: int) -> dict:
    ok = [r for r in results if r.get("status") == "ok"]
    windows = [(r["window_start"], r["window_end"]) for r in ok]
    overlap = overlap_fraction(windows)
    unit = ok[0]["unit"] if ok else None
    summary = {"n_gpus": n, "ok_gpus": len(ok), "unit": unit,
               "aggregate_peak": sum(r["peak"] for r in ok) if ok else None,
               "aggregate_median": sum(r["median"] for r in ok) if ok else None,
               "per_gpu_peak_min": min((r["peak"] for r in ok), default=None),
               "per_gpu_peak_max": max((r["peak"] for r in ok), default=None),
               "windows_overlap": overlap,
               "aggregate_valid": len(ok) == n and overlap >= OVERLAP_REQUIRED}
    summary["status"] = ("ok" if summary["aggregate_valid"] else
                         "error" if not ok else "partial")
    return summary


def parent_main(args, argv) -> dict:
    from torch.distributed import TCPStore
    import datetime
    store = TCPStore("127.0.0.1", 0, None, True,
                     timeout=datetime.timedelta(seconds=args.timeout), wait_for_workers=False)
    port = store.port
    forwarded = [a for a in argv if a not in ("--child",)]
    children = []
    for rank in range(args.gpus):
        cmd = [sys.executable, "-u", "-m", f"{PACKAGE}.replicas", *forwarded, "--child",
               "--rank", str(rank), "--store-port", str(port)]
        children.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                         text=True))
    deadline = time.time() + args.timeout
    logs = {}
    for rank, proc in enumerate(children):
        try:
            out, _ = proc.communicate(timeout=max(1.0, deadline - time.time()))
            logs[rank] = out[-4000:]
        except subprocess.TimeoutExpired:
            proc.kill()
            out, _ = proc.communicate()
            logs[rank] = (out or "")[-4000:]
    results = []
    for rank in range(args.gpus):
        key = f"result/{rank}"
        if store.check([key]):
            results.append(json.loads(store.get(key)))
        else:
            results.append({"rank": rank, "device": rank, "status": "error",
                            "reason": f"no result within {args.timeout:g} s (timeout or crash)",
                            "log_tail": logs.get(rank, "")[-1000:]})
    document = {"benchmark": "replicas", "probe": args.probe,
                "policy": "independent per-GPU replicas, host barrier before timing, "
                          "aggregate = sum of per-GPU peaks when all windows overlap >= 90%",
                "per_gpu": results, **aggregate(results, args.gpus)}
    if args.output:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(json.dumps(document, indent=2) + "\n")
    return document


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    args = build_parser().parse_args(argv)
    if args.child:
        return child_main(args)
    document = parent_main(args, argv)
    print(json.dumps({k: v for k, v in document.items() if k != "per_gpu"}))
    return 0 if document["status"] == "ok" else 1


if __name__ == "__main__":
    raise SystemExit(main())
