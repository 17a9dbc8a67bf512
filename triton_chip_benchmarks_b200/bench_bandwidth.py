#!/usr/bin/env python3
"""Peak device copy and read bandwidth on B200 through libtcb (sm_100a kernels).

Drop-in for the reference suite's bandwidth child (bench_bandwidth.py:113-249):
same flags, the same result rows and the same validation - a masked-tail
run first, a NaN sentinel before every measured copy, full-output equality
after it, and FP64 block-sum checks for the read pattern.  Copy traffic is
2 x buffer bytes; read traffic is buffer bytes + the FP32 sink.

Launch configurations are this build's own: the copy probe sweeps the
128-bit kernel (one CTA per piece of threads x 32 bytes) over threads per
CTA, and the bulk-copy-engine kernel over ring depths; the read probe sweeps
elements per CTA (--block-sizes) and warps.
"""

from __future__ import annotations

import argparse

import torch

from . import _native
from .runtime import (add_common_arguments, available_memory_bytes, emit_results,
                      emit_unsupported, measure, positive_int, setup_device)
from .validation import check_read

DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32,
          "u8": torch.uint8}
READ_DTYPES = {"fp32": _native.READ_FP32, "fp16": _native.READ_FP16,
               "bf16": _native.READ_BF16}
COPY_VARIANTS = {"ldg128": _native.COPY_LDG128, "bulk": _native.COPY_BULK}


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description=__doc__)
    add_common_arguments(parser)
    parser.add_argument("--mode", choices=["copy", "read", "all"], default="all",
                        help="Access patterns to measure separately (default: all)")
    parser.add_argument("--sizes-mib", type=positive_int, nargs="+",
                        default=[256, 512, 1024, 2048],
                        help="Size of EACH source/destination buffer in MiB")
    parser.add_argument("--dtype", choices=list(DTYPES), default="fp32",
                        help="Element type (u8 is copy-only)")
    parser.add_argument("--block-sizes", type=positive_int, nargs="+", default=[1024, 4096, 16384],
                        help="Elements per CTA of the read pattern (powers of two)")
    parser.add_argument("--num-warps", type=positive_int, nargs="+",
                        help="Warps per CTA of the read pattern (default: 4 8 16 32)")
    parser.add_argument("--copy-threads", type=positive_int, nargs="+", default=[512, 768, 1024],
                        help="Threads per CTA of the 128-bit copy kernel")
    parser.add_argument("--copy-variants", choices=list(COPY_VARIANTS), nargs="+",
                        default=list(COPY_VARIANTS), help="Copy kernels to measure")
    parser.add_argument("--bulk-stages", type=positive_int, nargs="+", default=[2, 4],
                        help="Shared-memory ring depths (32 KiB chunks) of the bulk-copy kernel")
    parser.add_argument("--copy-blocks-per-sm", type=positive_int, nargs="+", default=[4],
                        help="CTAs per SM of the bulk-copy kernel (grid = value x SMs); the "
                             "128-bit kernel launches one CTA per piece")
    parser.add_argument("--quick", action="store_true",
                        help="Smoke check: 8 MiB, one configuration per mode; not an HBM result")
    args = parser.parse_args(argv)
    if args.quick:
        args.sizes_mib, args.block_sizes, args.num_warps = [8], [1024], None
        args.copy_threads, args.copy_variants = [768], ["ldg128"]
        args.bulk_stages, args.copy_blocks_per_sm = [4], [4]
    if any(b & (b - 1) or b > 65536 or b < 256 for b in args.block_sizes):
        parser.error("--block-sizes must be powers of two in [256, 65536]")
    if args.num_warps is None:
        args.num_warps = [4] if args.quick else [4, 8, 16, 32]
    if any(w not in (4, 8, 16, 32) for w in args.num_warps):
        parser.error("--num-warps must be 4, 8, 16 or 32")
    if any(t % 32 or t > 1024 for t in args.copy_threads):
        parser.error("--copy-threads must be multiples of 32 up to 1024")
    return args


def copy_configs(args, sms: int):
    configs = []
    if "ldg128" in args.copy_variants:
        configs += [{"variant": "ldg128", "threads": t, "blocks": 0} for t in args.copy_threads]
    if "bulk" in args.copy_variants:
        configs += [{"variant": "bulk", "stages": st, "threads": 32, "blocks": per_sm * sms}
                    for per_sm in args.copy_blocks_per_sm for st in args.bulk_stages]
    return configs


def launch_copy(src, dst, config):
    knob = config["stages"] if config["variant"] == "bulk" else config["threads"]
    _native.copy(src, dst, src.numel() * src.element_size(), COPY_VARIANTS[config["variant"]],
                 config.get("blocks", 0), knob)


def launch_read(src, sink, block, warps, dtype_name):
    _native.read(src, READ_DTYPES[dtype_name], src.numel(), sink, block, warps * 32)


def main(argv=None):
    args = parse_args(argv)
    metadata = setup_device(args)
    device = torch.device("cuda", args.device)
    dtype = DTYPES[args.dtype]
    modes = ["copy", "read"] if args.mode == "all" else [args.mode]
    if args.dtype == "u8" and "read" in modes:
        if args.mode == "read":
            emit_unsupported("bandwidth", metadata, args,
                             "The read pattern sums floating-point elements; use fp32/fp16/bf16")
            return
        modes = ["copy"]
    element_size = torch.empty((), dtype=dtype).element_size()
    l2_bytes = metadata["l2_cache_bytes"]
    copies = copy_configs(args, metadata["sm_count"])
    reads = [(block, warps) for block in args.block_sizes for warps in args.num_warps]

    # Masked tails: sizes that do not fill a 16-byte vector or a block.
    for block, warps in reads or [(1024, 4)]:
        small = torch.randn(block + 17, device=device).to(dtype) if dtype != torch.uint8 else \
            torch.randint(0, 256, (block + 17,), device=device, dtype=dtype)
        if "copy" in modes:
            for config in copies:
                small_dst = torch.full_like(small, float("nan")) if dtype != torch.uint8 else \
                    torch.zeros_like(small)
                launch_copy(small, small_dst, config)
                if not torch.equal(small, small_dst):
                    raise AssertionError(f"Copy tail validation failed: {config}")
        if "read" in modes:
            sink = torch.full((-(-small.numel() // block),), float("nan"), device=device)
            launch_read(small, sink, block, warps, args.dtype)
            check_read(small, sink, block)
    print("Validation: masked tails passed; every measured output is checked in full.")
    print("Copy traffic = 2 * buffer bytes; read traffic = buffer bytes + FP32 sink. "
          "GB/s and TB/s are decimal; peak uses the shortest timed sample.")
    print("mode   buffer MiB   config            min ms   median ms   peak GB/s  median GB/s")
    rows = []
    for size_mib in args.sizes_mib:
        buffer_bytes = size_mib * 2**20
        n = buffer_bytes // element_size
        free = available_memory_bytes()
        sink_bytes = -(-n // min(args.block_sizes)) * 4 if "read" in modes else 0
        need = (2 if "copy" in modes else 1) * buffer_bytes + sink_bytes
        if free is not None and need + 512 * 2**20 > free:
            raise SystemExit(f"Insufficient free GPU memory for {size_mib} MiB buffers; "
                             "reduce --sizes-mib.")
        regime = ("unknown_l2" if not l2_bytes else
                  "larger_than_l2" if buffer_bytes >= 4 * l2_bytes else "cache_sensitive")
        eligible = regime == "larger_than_l2" and not args.quick
        if not eligible:
            reason = ("smoke mode" if args.quick else "L2 capacity is unavailable"
                      if not l2_bytes else "buffer is smaller than 4x L2")
            print(f"Note: {size_mib} MiB per buffer excluded from the HBM-sized peak summary: "
                  f"{reason}.")
        if dtype == torch.uint8:
            generator = torch.Generator(device=device).manual_seed(0)
            src = torch.randint(0, 256, (n,), device=device, dtype=dtype, generator=generator)
        else:
            src = torch.empty(n, device=device, dtype=dtype).normal_()
        dst = torch.empty_like(src) if "copy" in modes else None
        plans = ([("copy", c) for c in copies] if "copy" in modes else []) + \
                ([("read", r) for r in reads] if "read" in modes else [])
        for mode, config in plans:
            sink = None
            if mode == "copy":
                dst.fill_(float("nan") if dtype != torch.uint8 else 0)
                run = (lambda c=config: launch_copy(src, dst, c))
                run()
                if not torch.equal(src, dst):
                    raise AssertionError(f"Copy validation failed: size={size_mib}, {config}")
                correctness = {"correctness": "passed (full output and masked tail)"}
                write_bytes = buffer_bytes
                block, warps = config["threads"], config["threads"] // 32
                knob = config["stages"] if config["variant"] == "bulk" else config["threads"]
                label = (f"bulk/{config['stages']}st/{config['blocks']}b"
                         if config["variant"] == "bulk"
                         else f"ldg128/{config['threads']}t/pieces")
                info = _native.kernel_info(_native.FAMILY_COPY, COPY_VARIANTS[config["variant"]],
                                           knob)
            else:
                block, warps = config
                sink = torch.full((-(-n // block),), float("nan"), device=device)
                run = (lambda b=block, w=warps: launch_read(src, sink, b, w, args.dtype))
                run()
                correctness = check_read(src, sink, block)
                write_bytes = sink.numel() * sink.element_size()
                label = f"read/{block}e/{warps}w"
                info = _native.kernel_info(_native.FAMILY_READ, READ_DTYPES[args.dtype],
                                           warps * 32)
            timings = measure(run, args)
            traffic = buffer_bytes + write_bytes
            gbps = traffic / (timings["median_ms"] * 1e6)
            peak_gbps = traffic / (timings["min_ms"] * 1e6)
            row = {
                "mode": f"device_global_memory_{mode}", "pattern": mode, "dtype": args.dtype,
                "buffer_mib": size_mib, "buffer_bytes": buffer_bytes, "elements": n,
                "read_bytes": buffer_bytes, "write_bytes": write_bytes,
                "traffic_bytes": traffic, "block_size": block, "num_warps": warps,
                "kernel": label, "compiled": info,
                "cache_regime": regime, "peak_eligible": eligible, "smoke_only": args.quick,
                **timings, "gbps": gbps, "tbps": gbps / 1000,
                "peak_gbps": peak_gbps, "peak_tbps": peak_gbps / 1000, **correctness,
            }
            if mode == "copy":
                row["copy_variant"] = config["variant"]
                row["blocks"] = config["blocks"]
                if config["variant"] == "bulk":
                    row["bulk_ring_stages"] = config["stages"]
            rows.append(row)
            print(f"{mode:4s} {size_mib:11d}   {label:16s} {timings['min_ms']:9.4f} "
                  f"{timings['median_ms']:11.4f} {peak_gbps:11.2f} {gbps:12.2f}", flush=True)
            del sink
        del src, dst
        torch.cuda.empty_cache()
    eligible_rows = [row for row in rows if row["peak_eligible"]]
    for mode in modes:
        candidates = [row for row in (eligible_rows or rows) if row["pattern"] == mode]
        best = max(candidates, key=lambda row: row["peak_gbps"])
        label = "Best measured" if eligible_rows else "Best cache-sensitive/smoke"
        print(f"{label} {mode} bandwidth: {best['peak_gbps']:.2f} GB/s "
              f"({best['peak_tbps']:.3f} TB/s), {best['buffer_mib']} MiB/buffer, {best['kernel']}.")
    emit_results("bandwidth", metadata, args, rows)


if __name__ == "__main__":
    main()
