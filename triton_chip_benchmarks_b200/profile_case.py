#!/usr/bin/env python3
"""Run one probe configuration a fixed number of times (for profilers).

The sweep drivers time hundreds of launches through CUDA graphs; a profiler
capture wants a few plain launches of one configuration instead.  Each case
validates its first launch against the product's checks, then launches
`--launches` more times on the current stream and prints the device time of
those launches (CUDA events).

  python -m triton_chip_benchmarks_b200.profile_case copy --mib 1024 --variant bulk
  python -m triton_chip_benchmarks_b200.profile_case read --mib 1024 --block 4096
  python -m triton_chip_benchmarks_b200.profile_case tensor --dtype bf16 --tile 256x256x64
  python -m triton_chip_benchmarks_b200.profile_case vector --dtype fp32
  python -m triton_chip_benchmarks_b200.profile_case gemm --dtype fp4 --size 4096
"""

from __future__ import annotations

import argparse
import json

import torch

from . import _native
from .bench_tensor import NATIVE, STORAGE, VARIANTS, launch, peak_inputs, reference_output
from .bench_vector import make_inputs, native_dtype, validate
from .validation import validate_relative


def _time(fn, launches: int) -> float:
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(launches):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / max(launches, 1)


def case_copy(args) -> dict:
    n = args.mib << 20
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros_like(src)
    variant = {"ldg128": _native.COPY_LDG128, "bulk": _native.COPY_BULK}[args.variant]

    def run():
        _native.copy(src, dst, n, variant, args.blocks, args.threads)

    run()
    torch.cuda.synchronize()
    assert torch.equal(src, dst), "copy mismatch"
    ms = _time(run, args.launches)
    return {"case": "copy", "variant": args.variant, "bytes": n, "ms_per_launch": ms,
            "gbps": 2 * n / (ms * 1e6)}


def case_read(args) -> dict:
    """fp32 read-and-sum (tcb_read), the suite's read pattern; sink checked against torch."""
    n = (args.mib << 20) // 4
    src = torch.randn(n, device="cuda")
    blocks = -(-n // args.block)
    sink = torch.empty(blocks, device="cuda")

    def run():
        _native.read(src, _native.READ_FP32, n, sink, args.block, args.threads)

    run()
    torch.cuda.synchronize()
    expected = torch.nn.functional.pad(src.double(), (0, blocks * args.block - n))
    expected = expected.view(blocks, args.block).sum(1)
    assert torch.allclose(sink.double(), expected, rtol=1e-4, atol=1e-2), "read mismatch"
    ms = _time(run, args.launches)
    return {"case": "read", "bytes": 4 * n, "block": args.block, "threads": args.threads,
            "ms_per_launch": ms, "gbps": (4 * n + 4 * blocks) / (ms * 1e6)}


def case_tensor(args) -> dict:
    m, n, k = (int(v) for v in args.tile.split("x"))
    config = dict(block_m=m, block_n=n, block_k=k, chains=args.chains,
                  variant=VARIANTS[args.kernel])
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    blocks = sms * args.blocks_per_sm
    gen = torch.Generator().manual_seed(0)
    a, b, c, extras = peak_inputs(args.dtype, "baseline", blocks, config, torch.device("cuda"), gen)

    def run():
        launch(args.dtype, config, a, b, c, extras, blocks, args.blocks_per_sm, args.iterations)

    run()
    torch.cuda.synchronize()
    ref = reference_output(args.dtype, a, b, extras, args.iterations)
    validate_relative(c, ref, 1e-3 if args.dtype in ("bf16", "fp16", "tf32") else 0.0
                      if args.dtype in ("int8", "fp8", "fp4") else 1e-12)
    ms = _time(run, args.launches)
    ops = 2 * m * n * k * args.iterations * args.chains * blocks
    return {"case": "tensor", "dtype": args.dtype, "kernel": args.kernel, "tile": args.tile,
            "blocks": blocks, "iterations": args.iterations, "ms_per_launch": ms,
            "teraops": ops / (ms * 1e9), "storage": str(STORAGE[args.dtype]),
            "native_dtype": NATIVE[args.dtype]}


def case_vector(args) -> dict:
    ns = argparse.Namespace(dtype=args.dtype, int8_op=args.int8_op, inputs="baseline", seed=0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    blocks = sms * args.blocks_per_sm
    elements = blocks * args.threads * args.elems
    x, coeff = make_inputs(ns, elements, torch.device("cuda"))
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
    ms = _time(run, args.launches)
    per_update = 8 if args.dtype == "int8" and args.int8_op == "dp4a" else 2
    ops = per_update * 8 * elements * args.iterations
    return {"case": "vector", "dtype": args.dtype, "elements": elements,
            "iterations": args.iterations, "ms_per_launch": ms, "teraops": ops / (ms * 1e9)}


def case_gemm(args) -> dict:
    from .bench_tensor import GEMM_TOLERANCE, gemm_inputs, gemm_padded_k, gemm_reference
    m = n = k = args.size
    kp = gemm_padded_k(args.dtype, k)
    gen = torch.Generator().manual_seed(0)
    a, b, scales = gemm_inputs(args.dtype, m, n, k, torch.device("cuda"), gen)
    sa, sb = scales if scales is not None else (None, None)
    c = torch.empty((m, n), device="cuda",
                    dtype=torch.int32 if args.dtype == "int8" else
                    torch.float64 if args.dtype == "fp64" else torch.float32)

    def run():
        _native.gemm(NATIVE[args.dtype], a, b, c, m, n, kp, scale_a=sa, scale_b=sb)

    run()
    torch.cuda.synchronize()
    ref = gemm_reference(args.dtype, a, b)
    tol = GEMM_TOLERANCE[args.dtype]
    torch.testing.assert_close(c, ref, rtol=tol, atol=tol)
    ms = _time(run, args.launches)
    return {"case": "gemm", "dtype": args.dtype, "size": args.size, "ms_per_launch": ms,
            "teraops": 2 * m * n * k / (ms * 1e9)}


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = parser.add_subparsers(dest="case", required=True)
    p = sub.add_parser("copy")
    p.add_argument("--mib", type=int, default=1024)
    p.add_argument("--variant", choices=("ldg128", "bulk"), default="ldg128")
    p.add_argument("--threads", type=int, default=0)
    p.add_argument("--blocks", type=int, default=0)
    p.add_argument("--launches", type=int, default=3)
    p = sub.add_parser("read")
    p.add_argument("--mib", type=int, default=1024)
    p.add_argument("--block", type=int, default=4096, help="elements summed per CTA")
    p.add_argument("--threads", type=int, default=256)
    p.add_argument("--launches", type=int, default=3)
    p = sub.add_parser("tensor")
    p.add_argument("--dtype", default="bf16", choices=sorted(NATIVE))
    p.add_argument("--kernel", default="tcgen05", choices=("tcgen05", "dmma", "simt", "simt_reg"))
    p.add_argument("--tile", default="256x256x64")
    p.add_argument("--chains", type=int, default=1)
    p.add_argument("--blocks-per-sm", type=int, default=1)
    p.add_argument("--iterations", type=int, default=4096)
    p.add_argument("--launches", type=int, default=3)
    p = sub.add_parser("gemm")
    p.add_argument("--dtype", default="bf16", choices=("bf16", "fp16", "tf32", "fp32", "fp64", "int8", "fp8", "fp4"))
    p.add_argument("--size", type=int, default=4096)
    p.add_argument("--launches", type=int, default=3)
    p = sub.add_parser("vector")
    p.add_argument("--dtype", default="fp32", choices=("bf16", "fp16", "fp32", "fp64", "int8"))
    p.add_argument("--int8-op", default="dp4a", choices=("dp4a", "imad", "muladd"))
    p.add_argument("--blocks-per-sm", type=int, default=4)
    p.add_argument("--threads", type=int, default=256)
    p.add_argument("--elems", type=int, default=2)
    p.add_argument("--unroll", type=int, default=8)
    p.add_argument("--iterations", type=int, default=8192)
    p.add_argument("--launches", type=int, default=3)
    args = parser.parse_args(argv)
    torch.cuda.set_device(0)
    result = {"copy": case_copy, "read": case_read, "tensor": case_tensor,
              "vector": case_vector, "gemm": case_gemm}[args.case](args)
    print(json.dumps(result))


if __name__ == "__main__":
    main()
