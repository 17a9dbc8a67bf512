#!/usr/bin/env python3
"""Headline benchmark: device copy bandwidth of a 4 GiB buffer on B200.

Workload (the north-star configuration that fits one GPU): src and dst are
4 GiB contiguous uint8 buffers of seeded random bytes; one step is one copy
through libtcb's copy kernel; dst must equal src bit-exactly.  Bandwidth
counts read + write traffic, 2 x 4 GiB per step, in decimal GB/s.  The
buffers are 34x the 126 MB L2, so no cache flush is needed between steps.

`python bench.py --gpus N --steps K --warmup W` runs N independent replicas
(one process per GPU under torchrun, no collective on the data path; host
coordination over gloo), times exactly K steps with CUDA events between
barriers, takes the max over ranks and prints one JSON line on rank 0.
`--impl reference` times the reference's CPU path for the same workload
(a host copy of the buffer, restated in oracle/tcb_oracle.c) on rank 0.

After the copy's timed region the same line gains `rows`: every other
configuration of the benchmark's table (tensor probes, vector chains, the MX
FP4 8192^3 GEMM), each validated, timed with its own CUDA events and stamped
with the SM clock sampled while it ran (baseline_rows.py); `--no-rows` skips
them.
"""

from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
import sys
import time

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

BUFFER_BYTES = 4 * 2**30
METRIC = "memory_bandwidth (device copy, read+write bytes)"
UNIT = "GB/s"
WORKLOAD = "device copy of a 4 GiB uint8 buffer (src -> dst), seeded random bytes, bit-exact"


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--variant", choices=("ldg128", "bulk"), default="ldg128")
    parser.add_argument("--buffer-mib", type=int, default=BUFFER_BYTES >> 20,
                        help="buffer size (default: the 4 GiB workload; smaller only for profiling)")
    parser.add_argument("--threads", type=int, default=768, help="CTA size of the ldg128 kernel")
    parser.add_argument("--stages", type=int, default=0,
                        help="bulk kernel ring depth in 32 KiB chunks (0: library default)")
    parser.add_argument("--blocks", type=int, default=0,
                        help="CTAs (0: library default, one per piece for ldg128)")
    parser.add_argument("--e2e-chunk-mib", type=int, default=256,
                        help="chunk of the end-to-end pipeline (default: 256 MiB)")
    parser.add_argument("--e2e-steps", type=int, default=3,
                        help="steps of the host-buffer end-to-end leg")
    parser.add_argument("--cpu-seconds", type=float, default=10.0,
                        help="CPU-baseline sample duration")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-rows", action="store_true",
                        help="skip the per-configuration rows measured after the copy")
    return parser.parse_args()


# ---------------------------------------------------------------- plumbing
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_group(world: int):
    if world <= 1:
        return None
    import datetime
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    return dist


def barrier(dist):
    if dist is not None:
        dist.barrier()


def all_max(dist, value: float) -> float:
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_sum(dist, value: float) -> float:
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# --------------------------------------------------------------- baselines
def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


def ncu_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    path = REPO / "profiles" / "ncu_traffic.json"
    if not path.exists():
        return None
    table = json.loads(path.read_text())
    entry = table.get(kernel)
    return None if entry is None else float(entry["dram_bytes_per_launch"])


def cpu_copy_baseline(seconds: float, sample_bytes: int = BUFFER_BYTES) -> dict:
    """Host copy of the workload (oracle restatement), all host threads."""
    import numpy as np

    from oracle import native
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    src = rng.integers(0, 256, size=sample_bytes, dtype=np.uint8)
    dst = np.empty_like(src)
    native.copy(src, dst, threads)  # first touch
    copies, start = 0, time.perf_counter()
    used = threads
    while True:
        used = native.copy(src, dst, threads)
        copies += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            break
    if not np.array_equal(src[:1 << 20], dst[:1 << 20]):
        raise AssertionError("host copy mismatch")
    value = 2 * sample_bytes * copies / elapsed / 1e9
    return {"value": value, "unit": UNIT, "cores": used, "kind": "port",
            "sample": f"{copies} host copies of a {sample_bytes / 2**30:g} GiB uint8 buffer "
                      f"({elapsed:.1f} s, {used} threads, oracle/tcb_oracle.c oracle_copy)"}


# --------------------------------------------------------------- our impl
def run_ours(args):
    import torch

    from triton_chip_benchmarks_b200 import _native
    from triton_chip_benchmarks_b200.clocks import ClockSampler

    world, rank, local = dist_env()
    dist = init_group(world)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    variant = {"ldg128": _native.COPY_LDG128, "bulk": _native.COPY_BULK}[args.variant]
    threads = args.threads if args.variant == "ldg128" else args.stages

    nbytes = args.buffer_mib << 20
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=device, generator=gen)
    dst = torch.zeros_like(src)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream()

    def step():
        _native.copy(src, dst, nbytes, variant, args.blocks, threads, stream, status=status)

    def check(when):
        torch.cuda.synchronize()
        if int(status.item()) != 0:
            raise AssertionError(f"copy kernel reported {_native.strerror(int(status.item()))} "
                                 f"({when})")
        if not torch.equal(src, dst):
            raise AssertionError(f"copy validation failed: dst != src ({when})")

    step()
    check("first launch")
    dst.zero_()
    for _ in range(args.warmup):
        step()
    check("after warmup")
    # The timed steps must rebuild dst themselves: a step that did nothing would
    # leave these zeros behind and fail the check after the timed region.
    dst.zero_()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist)
    torch.cuda.synchronize()
    with ClockSampler(local) as sampler:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    clocks = sampler.summary()
    check("after the timed steps")
    barrier(dist)
    local_ms = start.elapsed_time(end)
    ms = all_max(dist, local_ms)
    ms_per_step = ms / args.steps
    traffic = 2 * nbytes
    value = world * traffic * args.steps / (ms / 1e3) / 1e9

    # End to end through the C ABI with host buffers: H2D of the step's input
    # from pinned memory, the copy kernel, D2H of the result, all timed.  The
    # buffer moves in chunks through three streams (host-to-device copy, copy
    # kernel, device-to-host copy) so the two PCIe directions run at once.
    e2e_value = None
    chunk = min(nbytes, args.e2e_chunk_mib << 20)
    if args.e2e_steps:
        host_src = src.cpu().pin_memory()
        host_dst = torch.empty_like(host_src).pin_memory()
        s_in, s_copy, s_out = (torch.cuda.Stream(device) for _ in range(3))
        bounds = [(a, min(nbytes, a + chunk)) for a in range(0, nbytes, chunk)]
        # Per chunk: input landed, kernel done (src chunk free again), output
        # read back (dst chunk free again).  A chunk is refilled only after the
        # previous step's kernel read it, and rewritten only after its read-back.
        landed = [torch.cuda.Event() for _ in bounds]
        copied = [torch.cuda.Event() for _ in bounds]
        drained = [torch.cuda.Event() for _ in bounds]

        def e2e_step(first):
            for i, (a, b) in enumerate(bounds):
                if not first:
                    s_in.wait_event(copied[i])
                with torch.cuda.stream(s_in):
                    src[a:b].copy_(host_src[a:b], non_blocking=True)
                landed[i].record(s_in)
                s_copy.wait_event(landed[i])
                if not first:
                    s_copy.wait_event(drained[i])
                _native.copy(src[a:b], dst[a:b], b - a, variant, args.blocks, threads, s_copy)
                copied[i].record(s_copy)
                s_out.wait_event(copied[i])
                with torch.cuda.stream(s_out):
                    host_dst[a:b].copy_(dst[a:b], non_blocking=True)
                drained[i].record(s_out)

        e2e_start = torch.cuda.Event(enable_timing=True)
        e2e_end = torch.cuda.Event(enable_timing=True)
        barrier(dist)
        torch.cuda.synchronize()
        e2e_start.record(stream)
        for side in (s_in, s_copy, s_out):
            side.wait_stream(stream)
        for k in range(args.e2e_steps):
            e2e_step(k == 0)
        for side in (s_in, s_copy, s_out):
            stream.wait_stream(side)
        e2e_end.record(stream)
        torch.cuda.synchronize()
        barrier(dist)
        e2e_ms = all_max(dist, e2e_start.elapsed_time(e2e_end))
        if not torch.equal(host_src, host_dst):
            raise AssertionError("end-to-end copy mismatch")
        e2e_value = world * traffic * args.e2e_steps / (e2e_ms / 1e3) / 1e9

        # What the link allows: each direction alone, the whole buffer in one
        # pinned copy, best of two.  With both directions at full rate at once
        # (PCIe is full duplex) an end-to-end step takes at least the slower
        # of the two, which bounds the end-to-end figure above.
        def one_way(copy):
            begin, finish = (torch.cuda.Event(enable_timing=True) for _ in range(2))
            begin.record(stream)
            copy()
            finish.record(stream)
            torch.cuda.synchronize()
            return begin.elapsed_time(finish)

        barrier(dist)
        h2d_ms = all_max(dist, min(one_way(lambda: src.copy_(host_src, non_blocking=True))
                                   for _ in range(2)))
        d2h_ms = all_max(dist, min(one_way(lambda: host_dst.copy_(dst, non_blocking=True))
                                   for _ in range(2)))
        ceiling = world * traffic / (max(h2d_ms, d2h_ms) / 1e3) / 1e9
        pcie = {"h2d_gbs": world * nbytes / (h2d_ms / 1e3) / 1e9,
                "d2h_gbs": world * nbytes / (d2h_ms / 1e3) / 1e9,
                "ceiling_gbs": ceiling, "pcie_frac": e2e_value / ceiling,
                "basis": "each direction timed alone (pinned, whole buffer, best of 2, max "
                         "over ranks); ceiling = both directions at once at those rates"}
        del host_src, host_dst

    # The north-star table's own configurations, measured after (outside) the
    # copy's timed region on every rank at once; rank 0 reports its rows and
    # the sum over ranks.
    rows = None
    if not args.no_rows:
        from triton_chip_benchmarks_b200 import baseline_rows
        del src, dst
        torch.cuda.empty_cache()
        barrier(dist)
        rows = baseline_rows.measure_rows(device, measured_peaks())
        for row in rows.values():
            total = all_sum(dist, row.get("value", 0.0) if row["status"] == "ok" else 0.0)
            if world > 1:
                row["aggregate_value"] = total
        barrier(dist)

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    peak_note = "of measured (MEASURED_PEAKS.json hbm_gbs, burst copy)"
    if peak is None:
        peak, peak_note = 6650.0, "of fallback"
    kernel_name = f"copy_{args.variant}"
    achieved = traffic / (local_ms / args.steps / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": ncu_traffic(kernel_name),
                "peak_source": peak_note, "algorithmic_bytes_per_launch": traffic,
                "kernel": kernel_name}
    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_copy_baseline(args.cpu_seconds)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded random bytes)",
        "config": {"workload": WORKLOAD if nbytes == BUFFER_BYTES else
                   f"profiling case: {args.buffer_mib} MiB copy (not the headline workload)",
                   "buffer_bytes": nbytes,
                   "bytes_per_step": traffic, "kernel": kernel_name,
                   "threads_per_cta": threads if args.variant == "ldg128" else 32,
                   "bulk_ring_stages": threads if args.variant == "bulk" else None,
                   "ctas": args.blocks or ("one per 24 KiB piece" if args.variant == "ldg128"
                                           and threads == 768 else "library default"),
                   "l2": "no flush: inputs (4 GiB) larger than the 126 MB L2",
                   "parallelism": f"replicas x{world} (no collective)"},
        "roofline": roofline, "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": nbytes,
                "d2h_bytes_per_step": nbytes, "steps": args.e2e_steps,
                "path": "pinned host -> device, tcb_copy, device -> pinned host, in "
                        f"{chunk >> 20} MiB chunks on three streams (both PCIe directions "
                        "at once)", **({"pcie": pcie} if e2e_value is not None else {})},
        "gpu_launches": args.steps, "clocks": clocks,
        "rows": rows,
    }
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import numpy as np

    from oracle import native
    threads = os.cpu_count() or 1
    nbytes = args.buffer_mib << 20
    rng = np.random.default_rng(1234)
    src = rng.integers(0, 256, size=nbytes, dtype=np.uint8)
    dst = np.zeros_like(src)
    for _ in range(args.warmup):
        native.copy(src, dst, threads)
    if not np.array_equal(src, dst):
        raise AssertionError("host copy mismatch")
    start = time.perf_counter()
    used = threads
    for _ in range(args.steps):
        used = native.copy(src, dst, threads)
    elapsed = time.perf_counter() - start
    traffic = 2 * nbytes
    value = traffic * args.steps / elapsed / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded random bytes)",
        "config": {"workload": WORKLOAD if nbytes == BUFFER_BYTES else
                   f"profiling case: {args.buffer_mib} MiB copy (not the headline workload)",
                   "buffer_bytes": nbytes, "bytes_per_step": traffic,
                   "parallelism": "host threads on rank 0"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": used, "kind": "port",
                         "sample": f"full {nbytes / 2**30:g} GiB buffer per step, {used} host threads "
                                   "(oracle/tcb_oracle.c oracle_copy)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
