#!/usr/bin/env python3
"""Typed vector FMA-chain throughput on B200 through libtcb (sm_100a kernels).

Drop-in for the reference suite's vector child (bench_vector.py:802-1575):
the same flags, statuses and result rows.  Eight independent chains per
element run x <- x*a + b_c in registers for --iterations steps:
bf16/fp16 as packed fma.rn.{bf16x2,f16x2}, fp32/fp64 as fma.rn.{f32,f64},
int8 as dp4a.s32.s32 (8 operations per update; --int8-op imad selects the
int32 wrap-around mad.lo.s32, --int8-op muladd the modulo-256 int8 state).
fp8 reports not_implemented and fp4 unsupported, as in the reference.

--inputs reference (default) uses the reference's exactly checkable value
sets (bench_vector.py:1191-1216); --inputs baseline uses x0 ~ U[0.5, 1),
a = 1 - 2**-10, b = 2**-10 (int: a = b = 1, int32 wrap) and checks every
element against a single-rounding replay of the recurrence.
"""

from __future__ import annotations

import argparse

import torch

from . import _native
from .runtime import (add_common_arguments, available_memory_bytes, emit_not_implemented,
                      emit_results, emit_unsupported, measure, positive_int, setup_device)
from .validation import (CHAINS, check_chain_exact, check_imad_output, check_int8_mul_add_output,
                         check_int8_output, check_output)

DEFAULT_ITERATIONS = 4096
DTYPES = ("bf16", "fp16", "fp32", "int8", "fp64", "fp8", "fp4")
TORCH_DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32,
                "fp64": torch.float64}
NATIVE_FLOAT = {"bf16": _native.V_BF16, "fp16": _native.V_FP16, "fp32": _native.V_FP32,
                "fp64": _native.V_FP64}
INT8_OPS = {"dp4a": _native.V_INT8_DP4A, "imad": _native.V_INT32_IMAD,
            "muladd": _native.V_INT8_MULADD}

FP8_VECTOR_REJECTION = (
    "This benchmark has no implemented and verified native FP8 vector arithmetic path; "
    "FP8 storage, conversions, or tensor instructions do not measure native FP8 vector "
    "throughput. This does not determine chip support")
FP4_VECTOR_REJECTION = (
    "FP4 (E2M1) is not an arithmetic element type for vector instructions: PTX has no "
    "E2M1 fused multiply-add, and PyTorch's float4_e2m1fn_x2 is a two-element container "
    "rather than a scalar type. FP4 storage, packing, conversions, or microscaled matrix "
    "instructions do not measure native FP4 vector throughput. This does not determine chip "
    "support; where a chip executes FP4 natively on its matrix unit, that rate is the "
    "tensor_fp4 metric")


def build_parser():
    parser = argparse.ArgumentParser(description=__doc__)
    add_common_arguments(parser)
    parser.add_argument("--dtype", choices=DTYPES, default="fp32",
                        help="Arithmetic type (default: fp32); fp8/fp4 emit a status JSON")
    parser.add_argument("--iterations", type=positive_int, default=DEFAULT_ITERATIONS,
                        help=f"Multiply-add iterations per accumulator (default: {DEFAULT_ITERATIONS})")
    parser.add_argument("--blocks-per-sm", type=positive_int, nargs="+",
                        help="Grid multipliers per SM (default: 8 16)")
    parser.add_argument("--block-sizes", type=positive_int, nargs="+",
                        help="Elements per CTA, powers of two (default: 256 512 1024 2048)")
    parser.add_argument("--num-warps", type=int, choices=[1, 2, 4, 8, 16, 32], nargs="+",
                        help="Warps per CTA (default: 4 8)")
    parser.add_argument("--unroll", type=int, choices=[1, 2, 4, 8, 16], nargs="+",
                        help="Loop unroll factors (default: 1 4 8 16)")
    parser.add_argument("--int8-op", choices=list(INT8_OPS), default="dp4a",
                        help="int8 arithmetic: dp4a (default, 8 ops/update), imad (int32 wrap), "
                             "muladd (int8 state mod 256)")
    parser.add_argument("--inputs", choices=("reference", "baseline"), default="reference",
                        help="Value set: the reference suite's exact sets, or the baseline "
                             "contraction x0~U[0.5,1), a=1-2**-10, b=2**-10")
    parser.add_argument("--seed", type=int, default=0, help="Input seed (default: 0)")
    parser.add_argument("--quick", action="store_true",
                        help="One smoke configuration; not a peak result")
    return parser


def configure_sweep(args):
    if args.quick:
        args.iterations = 32
        args.blocks_per_sm, args.block_sizes = [1], [256]
        args.num_warps, args.unroll = [4], [1]
    else:
        args.blocks_per_sm = args.blocks_per_sm or [8, 16]
        args.block_sizes = args.block_sizes or [256, 512, 1024, 2048]
        args.num_warps = args.num_warps or [4, 8]
        args.unroll = args.unroll or [1, 4, 8, 16]


def native_dtype(args) -> int:
    return INT8_OPS[args.int8_op] if args.dtype == "int8" else NATIVE_FLOAT[args.dtype]


def storage_dtype(args) -> torch.dtype:
    if args.dtype == "int8":
        return torch.int8 if args.int8_op == "muladd" else torch.int32
    return TORCH_DTYPES[args.dtype]


def ops_per_update(args) -> int:
    return 8 if args.dtype == "int8" and args.int8_op == "dp4a" else 2


def make_inputs(args, elements: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Initial states [8, elements] and coefficients [9] (a, b_0..b_7)."""
    gen = torch.Generator().manual_seed(args.seed)
    dtype = args.dtype
    if args.inputs == "baseline":
        if dtype == "int8":
            store = storage_dtype(args)
            lo, hi = (-128, 128) if store == torch.int8 else (-(2**31), 2**31)
            inputs = torch.randint(lo, hi, (CHAINS, elements), generator=gen, dtype=torch.int64)
            inputs = inputs.to(store)
            if args.int8_op == "dp4a":
                coeff = torch.tensor([0x01010101] + [1] * CHAINS, dtype=torch.int32)
            else:
                coeff = torch.tensor([1] + [1] * CHAINS, dtype=store)
        else:
            base = torch.rand((CHAINS, elements), generator=gen, dtype=torch.float64) * 0.5 + 0.5
            inputs = base.to(TORCH_DTYPES[dtype])
            coeff = torch.tensor([0.9990234375] + [0.0009765625] * CHAINS,
                                 dtype=TORCH_DTYPES[dtype])
        return inputs.to(device), coeff.to(device)
    # Reference value sets (bench_vector.py:1191-1216).
    if dtype == "int8" and args.int8_op == "muladd":
        inputs = torch.randint(-128, 128, (CHAINS, elements), generator=gen).to(torch.int8)
        coeff = torch.tensor([3] + [2 * c + 1 for c in range(CHAINS)], dtype=torch.int8)
    elif dtype == "int8" and args.int8_op == "imad":
        inputs = torch.randint(-(2**31), 2**31, (CHAINS, elements), generator=gen).to(torch.int32)
        coeff = torch.tensor([3] + [2 * c + 1 for c in range(CHAINS)], dtype=torch.int32)
    elif dtype == "int8":
        inputs = torch.randint(-(2**31), 2**31, (CHAINS, elements), generator=gen).to(torch.int32)
        packed = sum((v & 255) << s for v, s in zip((3, -2, 1, -1), (0, 8, 16, 24)))
        if packed >= 2**31:
            packed -= 2**32
        coeff = torch.tensor([packed] + list(range(1, CHAINS + 1)), dtype=torch.int32)
    elif dtype in ("fp16", "bf16"):
        inputs = (torch.randint(1, 8, (CHAINS, elements), generator=gen).double() / 8)
        inputs = inputs.to(TORCH_DTYPES[dtype])
        coeff = torch.tensor([-1.0] + [(i + 1) / 8 for i in range(CHAINS)],
                             dtype=TORCH_DTYPES[dtype])
    else:
        inputs = (torch.rand((CHAINS, elements), generator=gen, dtype=torch.float64) * 0.875
                  + 0.125).to(TORCH_DTYPES[dtype])
        coeff = torch.tensor([1.0 - 2.0**-14] + [(c + 1) * 2.0**-16 for c in range(CHAINS)],
                             dtype=TORCH_DTYPES[dtype])
    return inputs.to(device), coeff.to(device)


def validate(args, inputs, output, coeff, iterations) -> dict:
    if args.dtype == "int8":
        if args.int8_op == "dp4a":
            return check_int8_output(inputs, output, coeff, iterations)
        if args.int8_op == "muladd":
            return check_int8_mul_add_output(inputs, output, coeff, iterations)
        return check_imad_output(inputs, output, coeff, iterations)
    if args.inputs == "reference" or args.dtype == "fp64":
        return check_output(inputs, output, coeff, iterations, True)
    # Baseline 16/32-bit chains: every element replayed with one rounding per step.
    result = check_chain_exact(inputs, output, coeff, iterations)
    return {"correctness": "all elements bit-exact against a single-rounding FP64 replay",
            "max_abs_error": 0.0, "max_abs_tolerance": 0.0,
            "reference_device": str(output.device),
            "validation_recurrence": "per-step single-rounding replay", **result}


def sentinel(tensor: torch.Tensor, value) -> None:
    tensor.fill_(value)


def run_benchmark(args, metadata):
    device = torch.device("cuda", args.device)
    ndtype = native_dtype(args)
    store = storage_dtype(args)
    pack = 2 if args.dtype in ("bf16", "fp16") else 1
    per_update = ops_per_update(args)
    is_int = args.dtype == "int8"
    operation = {"dp4a": "DP4A", "imad": "IMAD_WRAP", "muladd": "INT8_MUL_ADD_MOD256"}[
        args.int8_op] if is_int else "FMA"
    unit = "TOPS" if is_int else "TFLOP/s"
    median_key, peak_key = ("tops", "peak_tops") if is_int else ("tflops", "peak_tflops")
    print(f"{args.dtype.upper()} vector: {CHAINS} independent {operation} chains, "
          f"{args.iterations} iterations; {per_update} operations per update; inputs={args.inputs}")
    print(f"blocks/SM  block  warps unroll regs  median_ms  median_{unit}  peak_{unit}")
    rows, excluded = [], []

    def exclude(kind, reason, **config):
        excluded.append({"status": kind, "reason": str(reason), **config})

    sms = metadata["sm_count"]
    for blocks_per_sm in args.blocks_per_sm:
        blocks = sms * blocks_per_sm
        for block_size in args.block_sizes:
            elements = blocks * block_size
            itemsize = torch.empty((), dtype=store).element_size()
            need = 2 * CHAINS * elements * itemsize
            free = available_memory_bytes()
            if free is not None and need > free * 0.5:
                raise SystemExit(f"Vector input/output need {need / 2**30:.2f} GiB; "
                                 "reduce --blocks-per-sm or --block-sizes")
            inputs, coeff = make_inputs(args, elements, device)
            coeff_host = coeff.cpu()
            output = torch.empty_like(inputs)
            for warps in args.num_warps:
                threads = warps * 32
                for unroll in args.unroll:
                    config = dict(blocks_per_sm=blocks_per_sm, block_size=block_size,
                                  num_warps=warps, unroll=unroll)
                    if block_size % threads or (block_size // threads) not in (1, 2, 4, 8, 16) \
                            or (block_size // threads) % pack:
                        exclude("configuration", f"{block_size} elements per CTA cannot be split "
                                f"into {threads} threads x 1-16 elements (pairs for 16-bit)",
                                **config)
                        continue
                    per_thread = block_size // threads
                    info = _native.kernel_info(_native.FAMILY_VECTOR, ndtype, threads, per_thread,
                                               unroll, int(ndtype in _native.COEFF_IN_REGISTERS))
                    if info["local_bytes_per_thread"]:
                        exclude("register_spills", f"local={info['local_bytes_per_thread']} B",
                                **config)
                        continue

                    coeff_arg = _native.vector_coefficients(ndtype, coeff, coeff_host)

                    def run(iterations=args.iterations, unroll_value=unroll,
                            per_thread=per_thread, threads=threads):
                        # Coefficients in registers or by value, per op.
                        _native.vector_chains(ndtype, inputs, output, coeff_arg, elements,
                                              iterations, blocks, threads, per_thread,
                                              unroll_value)

                    sentinel(output, -128 if store == torch.int8 else -(2**31) if is_int
                             else float("nan"))
                    run()
                    correctness = validate(args, inputs, output, coeff, args.iterations)
                    if is_int:
                        # Integer states have no NaN: re-run under a second poison,
                        # then an adjacent iteration count to catch an identity copy.
                        sentinel(output, 127 if store == torch.int8 else 2**31 - 1)
                        run()
                        validate(args, inputs, output, coeff, args.iterations)
                        sentinel(output, -128 if store == torch.int8 else -(2**31))
                        run(args.iterations + 1, 1)
                        validate(args, inputs, output, coeff, args.iterations + 1)
                        correctness["write_coverage_probe"] = "both poison values passed"
                        correctness["adjacent_iteration_probe"] = "all elements passed"
                    elif args.dtype in ("bf16", "fp16") and args.iterations % 2 == 0 \
                            and args.inputs == "reference":
                        sentinel(output, float("nan"))
                        run(args.iterations + 1, 1)
                        validate(args, inputs, output, coeff, args.iterations + 1)
                        correctness["odd_iteration_probe"] = "all elements passed"
                    timing = measure(run, args)
                    operations = per_update * CHAINS * elements * args.iterations
                    median = operations / (timing["median_ms"] * 1e9)
                    peak = operations / (timing["min_ms"] * 1e9)
                    rates = ({"counted_integer_ops": operations, "tops": median, "peak_tops": peak,
                              "throughput_unit": "TOPS", "ops_per_accumulator_update": per_update}
                             if is_int else
                             {"counted_flops": operations, "tflops": median, "peak_tflops": peak,
                              "throughput_unit": "TFLOP/s", "ops_per_accumulator_update": 2})
                    assembly = {
                        "registers_per_thread": info["registers_per_thread"],
                        "register_spills": info["local_bytes_per_thread"],
                        "assembly_check": (f"passed (source-level: {info['instruction']} written as "
                                           "inline PTX in the kernel; no tensor instructions)"),
                        "native_arithmetic_verified": True,
                        "ptx_arithmetic_instruction": info["instruction"],
                        "ptx_contains_tensor_instructions": False,
                    }
                    row = {
                        "status": "ok", "requested_dtype": args.dtype,
                        "dtype": str(store).removeprefix("torch."),
                        "input_storage_dtype": ("int8 packed in int32" if args.int8_op == "dp4a"
                                                else str(store).removeprefix("torch."))
                        if is_int else args.dtype,
                        "accumulator_dtype": ("int32" if store == torch.int32 else "int8")
                        if is_int else args.dtype,
                        "source_arithmetic_dtype": args.dtype,
                        "arithmetic_dtype": ("int8 products with int32 sum" if args.int8_op == "dp4a"
                                             else "int32" if args.int8_op == "imad" else "int8")
                        if is_int else args.dtype,
                        "includes_unpacking": False,
                        "operation": operation, "input_pattern": args.inputs,
                        "loop_structure": "strip_mined",
                        "coefficient_load": ("device_memory_to_registers"
                                             if ndtype in _native.COEFF_IN_REGISTERS
                                             else "kernel_parameter"),
                        "hardware_fusion_verified": not is_int,
                        "explicit_fma_supported": not is_int,
                        "dp4a_used": is_int and args.int8_op == "dp4a",
                        "packed_pairs": pack == 2,
                        "roundings_per_update": 1,
                        "accumulator_chains": CHAINS, "iterations": args.iterations,
                        "blocks_per_sm": blocks_per_sm, "blocks": blocks,
                        "block_size": block_size, "num_warps": warps, "unroll": unroll,
                        "elements_per_thread": per_thread,
                        "elements_per_chain": elements, "smoke_only": args.quick,
                        **rates, **timing, **correctness, **assembly,
                    }
                    rows.append(row)
                    print(f"{blocks_per_sm:9d} {block_size:6d} {warps:6d} {unroll:6d} "
                          f"{info['registers_per_thread']:4d} {timing['median_ms']:10.5f} "
                          f"{rates[median_key]:12.3f} {rates[peak_key]:11.3f}", flush=True)
            del inputs, output, coeff
    if not rows:
        reasons = "; ".join(dict.fromkeys(item["reason"] for item in excluded))
        raise RuntimeError(f"No vector configuration produced a valid measurement: {reasons}")
    best = max(rows, key=lambda row: row[peak_key])
    print(f"Peak measured {args.dtype.upper()} vector throughput: {best[peak_key]:.3f} {unit} "
          f"(median {best[median_key]:.3f} {unit}; blocks/SM={best['blocks_per_sm']}, "
          f"block={best['block_size']}, warps={best['num_warps']}, unroll={best['unroll']})")
    name = f"vector_{args.dtype}_" + ({"dp4a": "dot4", "imad": "imad", "muladd": "mul_add"}[
        args.int8_op] if is_int else "fma")
    emit_results(name, {**metadata, "vector_excluded_configurations": excluded}, args, rows)


def main(argv=None):
    parser = build_parser()
    args = parser.parse_args(argv)
    if args.block_sizes is not None and any(b & (b - 1) for b in args.block_sizes):
        parser.error("--block-sizes must contain only powers of two")
    if args.iterations >= 2**31 - 1:
        parser.error("--iterations must be less than 2**31 - 1")
    configure_sweep(args)
    metadata = setup_device(args)
    if args.dtype == "fp4":
        metadata["vector_fp4_capability_probe"] = {
            "ptx_e2m1_fma": False, "torch_fp4_container_dtype": str(
                getattr(torch, "float4_e2m1fn_x2", None)),
            "detail": "PTX defines no E2M1 multiply-add; FP4 executes only on tensor cores"}
        emit_unsupported("vector_fp4", metadata, args, FP4_VECTOR_REJECTION)
        return
    if args.dtype == "fp8":
        emit_not_implemented("vector_fp8", metadata, args, FP8_VECTOR_REJECTION)
        return
    run_benchmark(args, metadata)


if __name__ == "__main__":
    main()
