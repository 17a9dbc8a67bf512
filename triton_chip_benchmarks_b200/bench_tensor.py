#!/usr/bin/env python3
"""Resident-operand matrix peak throughput on B200 through libtcb (sm_100a kernels).

Drop-in for the reference suite's tensor child (bench_tensor.py:1311-1506):
the same flags, untimed precision probes, statuses and result rows.  Each
CTA keeps A [M x K] and B_c [K x N] (c < chains) resident and accumulates
A.B_c `--iterations` times; operations = 2*M*N*K*iterations*chains*blocks.

Execution units (no IEEE-FP32 tensor instruction exists on sm_100):
  bf16, fp16      tcgen05.mma kind::f16     -> FP32 in tensor memory
  tf32            tcgen05.mma kind::tf32    -> FP32 in tensor memory
  int8            tcgen05.mma kind::i8      -> INT32 in tensor memory
  fp8 (e4m3fn)    tcgen05.mma kind::f8f6f4  -> FP32 in tensor memory
  fp4 (MX E2M1)   tcgen05.mma kind::mxf4.block_scale, E8M0 scales in tensor memory
  fp64            mma.sync m16n8k4 f64 (tensor) and fma.rn.f64 (SIMT)
  fp32 (IEEE)     fma.rn.f32 register-blocked SIMT, labelled execution_kind=simt

--inputs reference (default) uses the reference's exact operand sets
(ternary/16; fp8 one-hot A rows; fp4 codes for +-0.5/+-1) and its
tolerance; --inputs baseline uses integers in [-3, 3] (scaled by 1/4 for
floats; fp4 draws all 16 E2M1 codes) with one accumulator chain, checked
exactly or within the stated relative tolerance.
"""

from __future__ import annotations

import argparse
import math

import torch

from . import _native
from .runtime import (add_common_arguments, available_memory_bytes, emit_not_implemented,
                      emit_results, emit_unsupported, measure, setup_device)
from .validation import (E2M1_VALUES, E8M0_UNIT_SCALE, FP4_PACKING_FACTOR, MX_GROUP_SIZE,
                         accumulator_name, decode_e2m1, pack_e2m1_pairs, reference_product,
                         validate_peak, validate_relative)


class TensorUnsupportedError(RuntimeError):
    """The requested format or its required execution precision is unavailable."""


NATIVE = {"bf16": _native.T_BF16, "fp16": _native.T_FP16, "tf32": _native.T_TF32,
          "fp32": _native.T_FP32, "fp64": _native.T_FP64, "int8": _native.T_INT8,
          "fp8": _native.T_FP8E4M3, "fp4": _native.T_MXF4}
STORAGE = {"bf16": torch.bfloat16, "fp16": torch.float16, "tf32": torch.float32,
           "fp32": torch.float32, "fp64": torch.float64, "int8": torch.int8,
           "fp8": torch.float8_e4m3fn, "fp4": torch.uint8}
VARIANT_NAMES = {_native.TV_TCGEN05: "tcgen05", _native.TV_DMMA: "dmma", _native.TV_SIMT: "simt",
                 _native.TV_SIMT_REG: "simt_reg"}
VARIANTS = {name: variant for variant, name in VARIANT_NAMES.items()}
# Relative tolerance of the baseline operand sets (exact results pass trivially).
BASELINE_RTOL = {"bf16": 1e-3, "fp16": 1e-3, "tf32": 1e-3, "fp32": 1e-5, "fp64": 1e-12,
                 "int8": 0.0, "fp8": 0.0, "fp4": 0.0}


def math_key(args) -> str:
    """Row key: fp32 with TF32 input precision runs as tf32."""
    return "tf32" if args.dtype == "fp32" and args.input_precision == "tf32" else args.dtype


def rates(operation_count: int, timing: dict, dtype: str) -> dict:
    median = operation_count / (timing["median_ms"] * 1e9)
    peak = operation_count / (timing.get("min_ms", timing["median_ms"]) * 1e9)
    integer = dtype == "int8"
    return {"operation_count": operation_count,
            "operation_type": "integer" if integer else "floating_point",
            "throughput_unit": "TOPS" if integer else "TFLOP/s",
            "median_teraops_per_second": median, "peak_teraops_per_second": peak,
            **({"integer_ops": operation_count, "tops": median, "peak_tops": peak}
               if integer else {"flops": operation_count, "tflops": median, "peak_tflops": peak})}


def precision_descriptor(dtype: str, dot_input_precision: str | None) -> dict:
    storage = "fp32" if dtype == "fp32" else ("e4m3fn" if dtype == "fp8" else
                                              "e2m1" if dtype == "fp4" else dtype)
    if dtype == "fp32":
        math_mode = "tf32" if dot_input_precision == "tf32" else "ieee_fp32"
    elif dtype == "fp4":
        math_mode = "mxfp4_e2m1"
    else:
        math_mode = dtype
    descriptor = {"input_format": storage, "input_storage_dtype": storage,
                  "dot_input_precision": dot_input_precision, "math_mode": math_mode}
    if dtype == "fp4":
        descriptor.update({
            "container_dtype": "uint8", "elements_per_container": FP4_PACKING_FACTOR,
            "scale_format": "e8m0", "scale_group_size": MX_GROUP_SIZE,
            "scale_value": "2**0 (E8M0 code 127) for every group", "microscaled": True,
            "dot_operation": "tcgen05.mma kind::mxf4.block_scale"})
    return descriptor


def normalize_precision_args(parser, args) -> None:
    args.requested_dtype = args.dtype
    if args.dtype == "tf32":
        if args.input_precision not in (None, "tf32"):
            parser.error("--dtype tf32 cannot use --input-precision ieee")
        args.dtype, args.input_precision = "fp32", "tf32"
    elif args.dtype == "fp32":
        args.input_precision = args.input_precision or "ieee"
    elif args.input_precision is not None:
        parser.error("--input-precision is only valid with --dtype fp32")


# ------------------------------------------------------------------ configs
def default_k(key: str, inputs: str) -> int:
    if inputs == "baseline":
        return {"bf16": 64, "fp16": 64, "tf32": 32, "fp32": 32, "fp64": 32, "int8": 128,
                "fp8": 128, "fp4": 256}[key]
    return {"bf16": 32, "fp16": 32, "tf32": 32, "fp32": 32, "fp64": 16, "int8": 64,
            "fp8": 64, "fp4": 128}[key]


def peak_configs(key: str, inputs: str) -> list[dict]:
    """This build's tile sweep: (variant, tile_m, tile_n, tile_k, chains)."""
    k = default_k(key, inputs)
    chains = 1 if inputs == "baseline" else 2
    configs = []
    if key == "fp32":
        tiles = [(_native.TV_SIMT, 128, 128), (_native.TV_SIMT, 256, 256),
                 (_native.TV_SIMT_REG, 64, 64), (_native.TV_SIMT_REG, 128, 128),
                 (_native.TV_SIMT_REG, 256, 256)]
        if inputs == "reference":  # the reference's IEEE FP32 tiles, bench_tensor.py:499-503
            tiles += [(_native.TV_SIMT_REG, 32, 32), (_native.TV_SIMT_REG, 32, 64),
                      (_native.TV_SIMT_REG, 64, 32)]
    elif key == "fp64":
        tiles = [(_native.TV_DMMA, 128, 128), (_native.TV_DMMA, 256, 256),
                 (_native.TV_SIMT, 128, 128), (_native.TV_SIMT, 256, 256),
                 (_native.TV_SIMT_REG, 64, 64), (_native.TV_SIMT_REG, 256, 256)]
        if inputs == "reference":  # the reference's FP64 tiles, bench_tensor.py:497-498
            tiles += [(_native.TV_SIMT_REG, 32, 32), (_native.TV_SIMT_REG, 32, 64)]
    else:
        tiles = [(_native.TV_TCGEN05, 128, 128), (_native.TV_TCGEN05, 128, 256),
                 (_native.TV_TCGEN05, 256, 256)]
    # The reference's K and twice it: a deeper resident K amortizes the per-tile
    # staging and epilogue over more MMAs without changing what is counted.
    ks = [k] if key in ("fp32", "fp64") or inputs == "baseline" else [k, 2 * k]
    for kk in ks:
        for variant, m, n in tiles:
            configs.append(dict(block_m=m, block_n=n, block_k=kk, chains=chains,
                                variant=variant, kernel=VARIANT_NAMES[variant],
                                num_warps=4 if variant == _native.TV_TCGEN05 else 8,
                                num_stages=1))
    return configs


# ------------------------------------------------------------------- inputs
def _ternary16(shape, gen, dtype):
    return (torch.randint(-1, 2, shape, generator=gen).double() / 16).to(dtype)


def peak_inputs(key: str, inputs: str, blocks: int, config: dict, device, gen):
    """A [blocks,M,K], B [chains,blocks,N,K] (K contiguous), C, and FP4 extras."""
    m, n, k, chains = config["block_m"], config["block_n"], config["block_k"], config["chains"]
    dtype = STORAGE[key]
    extras = None
    if key == "fp4":
        if inputs == "baseline":
            a_codes = torch.randint(0, 16, (blocks, m, k), generator=gen, dtype=torch.uint8)
            b_codes = torch.randint(0, 16, (chains, blocks, n, k), generator=gen, dtype=torch.uint8)
        else:
            palette = torch.tensor([1, 2, 9, 10], dtype=torch.uint8)
            a_codes = palette[torch.randint(4, (blocks, m, k), generator=gen)]
            b_codes = palette[torch.randint(4, (chains, blocks, n, k), generator=gen)]
        a = pack_e2m1_pairs(a_codes).to(device)
        b = pack_e2m1_pairs(b_codes).to(device)
        sa = torch.full((blocks, m, k // MX_GROUP_SIZE), E8M0_UNIT_SCALE, dtype=torch.uint8,
                        device=device)
        sb = torch.full((blocks, n, k // MX_GROUP_SIZE), E8M0_UNIT_SCALE, dtype=torch.uint8,
                        device=device)
        extras = (sa, sb)
    elif inputs == "baseline":
        ints_a = torch.randint(-3, 4, (blocks, m, k), generator=gen)
        ints_b = torch.randint(-3, 4, (chains, blocks, n, k), generator=gen)
        if key == "int8":
            a, b = ints_a.to(torch.int8), ints_b.to(torch.int8)
        else:
            a = (ints_a.double() / 4).to(dtype)
            b = (ints_b.double() / 4).to(dtype)
        a, b = a.to(device), b.to(device)
    elif key == "fp8":
        # One-hot A rows keep every dot at +-1/256 (bench_tensor.py:651-660).
        a = torch.zeros((blocks, m, k), dtype=torch.float64)
        a.scatter_(2, torch.randint(k, (blocks, m, 1), generator=gen), 1 / 16)
        b = (torch.randint(0, 2, (chains, blocks, n, k), generator=gen).double() * 2 - 1) / 16
        a, b = a.to(dtype).to(device), b.to(dtype).to(device)
    elif key == "int8":
        a = torch.randint(-1, 2, (blocks, m, k), generator=gen).to(torch.int8).to(device)
        b = torch.randint(-1, 2, (chains, blocks, n, k), generator=gen).to(torch.int8).to(device)
    else:
        a = _ternary16((blocks, m, k), gen, dtype).to(device)
        b = _ternary16((chains, blocks, n, k), gen, dtype).to(device)
    out_dtype = (torch.int32 if key == "int8" else torch.float64 if key == "fp64"
                 else torch.float32)
    c = torch.empty((chains, blocks, m, n), dtype=out_dtype, device=device)
    return a, b, c, extras


def reference_output(key, a, b, extras, iterations):
    """Exact A.B_c^T * iterations for every chain and block."""
    if key == "fp4":
        product = torch.matmul(decode_e2m1(a), decode_e2m1(b).transpose(-1, -2))
        return (product * iterations).float()
    ref = reference_product(a, b)
    if ref.dtype == torch.int32:
        return ref * iterations
    return ref * iterations


def fp4_exactness(a, b, iterations) -> float:
    """Largest |A.B| entry; 4096*S stays exact in FP32 only while |S|*iterations*4 < 2**24."""
    return torch.matmul(decode_e2m1(a), decode_e2m1(b).transpose(-1, -2)).abs().max().item()


def launch(key, config, a, b, c, extras, blocks, blocks_per_sm, iterations, status=None):
    sa, sb = extras if extras is not None else (None, None)
    _native.tensor_peak(NATIVE[key], config["variant"], a, b, c, blocks=blocks,
                        blocks_per_sm=blocks_per_sm, tile_m=config["block_m"],
                        tile_n=config["block_n"], tile_k=config["block_k"],
                        chains=config["chains"], iterations=iterations, scale_a=sa, scale_b=sb,
                        status=status)


def kernel_info(key, config, blocks_per_sm) -> dict:
    return _native.kernel_info(_native.FAMILY_TENSOR, NATIVE[key], config["variant"],
                               config["block_m"], config["block_n"], config["block_k"],
                               config["chains"], blocks_per_sm)


# ------------------------------------------------------------------ probes
def validate_fp32_precision(device, precision: str) -> dict:
    """IEEE and TF32 give different exact answers (bench_tensor.py:675-714).

    A holds 1+2**-12 (not TF32-representable), with markers 1+2**-9 and
    2**20 in row 0; B is the identity.  IEEE returns A; TF32 returns 1.0
    except at the two markers.
    """
    tail, mantissa, exponent = 1.0 + 2.0**-12, 1.0 + 2.0**-9, 2.0**20
    m, n, k = 128, 128, 32
    if precision == "tf32":
        key, config = "tf32", dict(block_m=128, block_n=32, block_k=32, chains=1,
                                   variant=_native.TV_TCGEN05)
        n = 32
    else:
        key, config = "fp32", dict(block_m=128, block_n=128, block_k=32, chains=1,
                                   variant=_native.TV_SIMT)
    a = torch.full((1, m, k), tail, dtype=torch.float32, device=device)
    a[0, 0, 1] = mantissa
    a[0, 0, 2] = exponent
    b = torch.eye(n, k, dtype=torch.float32, device=device).unsqueeze(0).unsqueeze(0)
    c = torch.full((1, 1, m, n), float("nan"), dtype=torch.float32, device=device)
    launch(key, config, a, b, c, None, 1, 1, 1)
    expected = torch.zeros((m, n), dtype=torch.float32, device=device)
    expected[:, :k] = a[0] if precision == "ieee" else 1.0
    if precision == "tf32":
        expected[0, 1], expected[0, 2] = mantissa, exponent
    error = (c[0, 0] - expected).abs().max().item()
    if error != 0.0 or not torch.isfinite(c).all():
        raise TensorUnsupportedError(
            f"The matrix path did not honour input precision {precision!r}: probe expected "
            f"{expected[0, 0].item()}, observed {c[0, 0, 0, 0].item()}, max error {error}")
    return {"passed": True, "max_abs_error": error,
            "probe_values": [tail, mantissa, exponent], "kernel_mode": "peak",
            "description": "A contains 1+2^-12, 1+2^-9 and 2^20; B=identity; distinguishes "
                           "IEEE, TF32, BF16 and FP16"}


def validate_fp64_precision(device, variant: int) -> dict:
    """FP64 exactness and row placement (bench_tensor.py:717-757)."""
    m = n = 128
    k = 16
    a = torch.full((1, m, k), 1.0 + 2.0**-40, dtype=torch.float64, device=device)
    a[0, :, 0] = torch.arange(1, m + 1, dtype=torch.float64, device=device)
    b = torch.eye(n, k, dtype=torch.float64, device=device).unsqueeze(0).unsqueeze(0)
    c = torch.full((1, 1, m, n), float("nan"), dtype=torch.float64, device=device)
    config = dict(block_m=m, block_n=n, block_k=k, chains=1, variant=variant)
    launch("fp64", config, a, b, c, None, 1, 1, 1)
    expected = torch.zeros((m, n), dtype=torch.float64, device=device)
    expected[:, :k] = a[0]
    error = (c[0, 0] - expected).abs().max().item()
    if error != 0.0 or not torch.isfinite(c).all():
        rows_a = sorted(map(tuple, c[0, 0].cpu().tolist()))
        rows_e = sorted(map(tuple, expected.cpu().tolist()))
        detail = ("the returned rows are a permutation of the correct rows"
                  if rows_a == rows_e else f"probe error={error}")
        raise TensorUnsupportedError(f"FP64 matrix path is not exact: {detail}")
    return {"passed": True, "max_abs_error": error, "kernel_mode": "peak",
            "kernel": VARIANT_NAMES[variant],
            "description": "FP64 (1+2^-40) with a per-row marker times identity; rejects FP32 "
                           "fallback and permuted output rows"}


def validate_gemm_precision(device, key: str) -> dict:
    """The fp32/tf32 and fp64 precision probes through the GEMM kernel itself.

    The reference runs the same probes on its GEMM kernel in --mode gemm
    (bench_tensor.py:675-714, 717-757 with mode "gemm"): 32 x 32 x 32, B the
    identity.  fp32/tf32: A holds 1+2**-12 with markers 1+2**-9 and 2**20 in
    row 0; fp64: A holds 1+2**-40 with a per-row marker in column 0.
    """
    size = 32
    if key == "fp64":
        a = torch.full((size, size), 1.0 + 2.0**-40, dtype=torch.float64, device=device)
        a[:, 0] = torch.arange(1, size + 1, dtype=torch.float64, device=device)
        expected = a.clone()
        values = [1.0 + 2.0**-40]
    else:
        tail, mantissa, exponent = 1.0 + 2.0**-12, 1.0 + 2.0**-9, 2.0**20
        a = torch.full((size, size), tail, dtype=torch.float32, device=device)
        a[0, 1], a[0, 2] = mantissa, exponent
        expected = a.clone()
        if key == "tf32":
            expected.fill_(1.0)
            expected[0, 1], expected[0, 2] = mantissa, exponent
        values = [tail, mantissa, exponent]
    b = torch.eye(size, dtype=a.dtype, device=device)
    c = torch.full((size, size), float("nan"), dtype=a.dtype, device=device)
    _native.gemm(NATIVE[key], a, b, c, size, size, size)
    torch.cuda.synchronize(device)
    error = (c - expected).abs().max().item()
    if error != 0.0 or not torch.isfinite(c).all():
        if key == "fp64":
            permuted = sorted(map(tuple, c.cpu().tolist())) == sorted(map(tuple, expected.cpu().tolist()))
            raise TensorUnsupportedError(
                "FP64 GEMM is not exact: " + ("the returned rows are a permutation of the "
                                              "correct rows" if permuted else f"probe error={error}"))
        raise TensorUnsupportedError(
            f"The GEMM did not honour input precision {key!r}: probe expected "
            f"{expected[0, 0].item()}, observed {c[0, 0].item()}, max error {error}")
    description = ("FP64 (1+2^-40) with a per-row marker times identity; rejects FP32 fallback "
                   "and permuted output rows" if key == "fp64" else
                   "A contains 1+2^-12, 1+2^-9 and 2^20; B=identity; distinguishes IEEE, TF32, "
                   "BF16 and FP16")
    return {"passed": True, "max_abs_error": error, "probe_values": values,
            "kernel_mode": "gemm", "description": description}


def validate_fp8_storage(device) -> dict:
    probe = torch.tensor([1 / 16, -1 / 16, 1.0], dtype=torch.float32, device=device)
    restored = probe.to(torch.float8_e4m3fn).float()
    error = (restored - probe).abs().max().item()
    if error != 0.0:
        raise TensorUnsupportedError(f"FP8 E4M3FN storage round-trip error={error}")
    return {"passed": True, "max_abs_error": error, "probe_values": [1 / 16, -1 / 16, 1.0],
            "description": "FP8 E4M3FN storage round-trip of exactly representable values"}


def validate_fp4_arithmetic(device) -> dict:
    """Exact E2M1 products, then a doubled A scale must double C (bench_tensor.py:829-886)."""
    gen = torch.Generator().manual_seed(0)
    config = dict(block_m=128, block_n=128, block_k=128, chains=2, variant=_native.TV_TCGEN05)
    a, b, c, (sa, sb) = peak_inputs("fp4", "reference", 1, config, device, gen)
    launch("fp4", config, a, b, c, (sa, sb), 1, 1, 1)
    reference = reference_output("fp4", a, b, None, 1).double()
    error = (c.double() - reference).abs().max().item()
    if error != 0.0:
        raise TensorUnsupportedError("MX FP4 path is not exact: max_abs_error="
                                     f"{error} against the exact E2M1 reference")
    doubled = torch.empty_like(c)
    launch("fp4", config, a, b, doubled, (torch.full_like(sa, E8M0_UNIT_SCALE + 1), sb), 1, 1, 1)
    scale_error = (doubled.double() - 2.0 * reference).abs().max().item()
    if scale_error != 0.0:
        raise TensorUnsupportedError("MX FP4 path did not apply the E8M0 scale: raising A's "
                                     f"scale to 2**1 left max_abs_error={scale_error}")
    return {"passed": True, "kernel_mode": "peak", "probed_tile": "128x128x128",
            "max_abs_error": 0.0, "scale_sensitivity_verified": True,
            "description": "MX FP4 (E2M1 packed two per uint8, E8M0 unit scales) exact-product "
                           "and scale-application probe"}


# ------------------------------------------------------------------- audit
EXPECTED_INSTRUCTION = {
    "bf16": "kind::f16 (bf16 x bf16 -> f32)", "fp16": "kind::f16 (f16 x f16 -> f32)",
    "tf32": "kind::tf32", "int8": "kind::i8 (s8 x s8 -> s32)",
    "fp8": "kind::f8f6f4 (e4m3 x e4m3 -> f32)", "fp4": "kind::mxf4.block_scale",
}


def compiled_info(key: str, info: dict, verified_by_probe: bool) -> dict:
    """Audit fields from the kernel's source instruction table and probes.

    The instruction is the one the kernel's source writes as inline PTX;
    compiled PTX/SASS is never read.  A tensor-core kernel whose source
    instruction does not match the requested format is rejected.
    """
    instruction = info["instruction"]
    tensor = info["execution_kind"] == "tensor"
    if key in EXPECTED_INSTRUCTION and EXPECTED_INSTRUCTION[key] not in instruction:
        raise TensorUnsupportedError(f"Cannot verify native {key} MMA: kernel writes {instruction}")
    if key == "fp32" and tensor:
        raise TensorUnsupportedError("Requested IEEE FP32 but the kernel uses a tensor instruction")
    return {
        "registers_per_thread": info["registers_per_thread"],
        "spill_count": info["local_bytes_per_thread"],
        "shared_memory_bytes": info["static_smem_bytes"] + info["dynamic_smem_bytes"],
        "assembly_audit": "verified", "execution_kind": "tensor" if tensor else "simt",
        "instruction_precision_verified": True if key not in ("fp32", "fp64", "fp4")
        else verified_by_probe,
        "native_tensor_verified": tensor,
        "assembly_audit_note": (
            "instruction taken from the kernel source (inline PTX); compiled PTX/SASS is not "
            "inspected" + ("" if tensor else f"; {key.upper()} execution is scalar FMA, "
                           "no native tensor MMA")),
        "tensor_instruction_types": [instruction] if tensor else [],
        "static_tensor_instruction_count": 1 if tensor else 0,
        "fp32_fma_instruction_types": [instruction] if instruction == "fma.rn.f32" else [],
        "fp64_fma_instruction_types": [instruction] if instruction == "fma.rn.f64" else [],
        "static_fp32_fma_instruction_count": 1 if instruction == "fma.rn.f32" else 0,
    }


# ------------------------------------------------------------------- sweep
def run_peak(args, metadata) -> None:
    key = math_key(args)
    device = torch.device("cuda", args.device)
    sms = metadata["sm_count"]
    candidates = peak_configs(key, args.inputs)
    if args.tiles:
        wanted = {tuple(int(v) for v in t.split("x")) for t in args.tiles}
        candidates = [c for c in candidates if (c["block_m"], c["block_n"]) in wanted
                      or (c["block_m"], c["block_n"], c["block_k"]) in wanted]
    if args.block_k:
        candidates = [{**c, "block_k": args.block_k} for c in candidates]
    if args.quick:
        candidates = candidates[:1]
        args.blocks_per_sm = [1]
        args.iterations = min(args.iterations, 64)
    accumulator = accumulator_name(key)
    unit = "TOPS" if key == "int8" else "TFLOP/s"
    print(f"\nMatrix peak: resident {key} operands, {candidates[0]['chains'] if candidates else 0} "
          f"{accumulator.upper()} accumulator chain(s), inputs={args.inputs}")
    print(f"Iterations={args.iterations}; operations=2*tile_M*tile_N*tile_K*iterations*chains*blocks")
    print(f"  kernel   tile M/N/K  chains blocks/SM   median ms   min ms  median {unit}  peak {unit}  regs")
    rows = []
    gen = torch.Generator().manual_seed(args.seed)
    for config in candidates:
        for blocks_per_sm in args.blocks_per_sm:
            blocks = blocks_per_sm * sms
            m, n, k = config["block_m"], config["block_n"], config["block_k"]
            base = {"mode": "peak", "dtype": key, "config": config, "blocks_per_sm": blocks_per_sm}
            try:
                info = kernel_info(key, config, blocks_per_sm)
            except _native.TcbError as exc:
                if exc.is_resource or exc.is_capability or exc.status == _native.ERR_INVALID_ARGUMENT:
                    rows.append({**base, "status": "skipped", "reason": str(exc)})
                    continue
                raise
            if info["local_bytes_per_thread"]:
                rows.append({**base, "status": "skipped", "reason": "configuration spills registers"})
                continue
            free = available_memory_bytes()
            need = blocks * (m * k + 2 * k * n + 8 * m * n) * 8
            if free is not None and need > free * 0.8:
                raise RuntimeError("Peak validation exceeds available memory; reduce --blocks-per-sm")
            a, b, c, extras = peak_inputs(key, args.inputs, blocks, config, device, gen)
            if key == "fp4" and args.inputs == "baseline":
                largest = fp4_exactness(a, b, args.iterations)
                if largest * args.iterations * 4 >= 2**24:
                    raise RuntimeError(f"FP4 operand draw has |A.B| up to {largest}; "
                                       f"{args.iterations}x it is not exact in FP32")
            c.fill_(-2**31 if key == "int8" else float("nan"))
            status = torch.zeros(1, dtype=torch.int32, device=device)
            try:
                launch(key, config, a, b, c, extras, blocks, blocks_per_sm, args.iterations, status)
            except _native.TcbError as exc:
                if exc.is_resource:
                    rows.append({**base, "status": "skipped", "reason": str(exc)})
                    continue
                if exc.is_capability:
                    rows.append({**base, "status": "unsupported", "reason": str(exc)})
                    continue
                raise
            torch.cuda.synchronize()
            if int(status.item()) != 0:
                raise RuntimeError(f"device-side wait failed: {_native.strerror(int(status.item()))}")
            reference = reference_output(key, a, b, extras, args.iterations)
            if args.inputs == "baseline":
                correctness = validate_relative(c, reference, BASELINE_RTOL[key])
            else:
                correctness = validate_peak(c, reference.to(c.dtype), key, k, args.iterations)
            del reference
            audit = compiled_info(key, info, bool(metadata.get("tensor_precision_probe")
                                                  or metadata.get("tensor_dot_lowering_probe")))
            timing = measure(lambda: launch(key, config, a, b, c, extras, blocks, blocks_per_sm,
                                            args.iterations, status), args)
            torch.cuda.synchronize()
            if int(status.item()) != 0:
                raise RuntimeError(f"device-side wait failed: {_native.strerror(int(status.item()))}")
            operations = 2 * m * n * k * args.iterations * config["chains"] * blocks
            rate = rates(operations, timing, key)
            descriptor = precision_descriptor(args.dtype, args.input_precision)
            if key in ("fp32", "fp64"):
                kind = (f"{descriptor['math_mode']}_tensor_peak" if audit["native_tensor_verified"]
                        else f"{descriptor['math_mode']}_matrix_throughput")
            else:
                kind = "native_tensor_peak"
            row = {
                **base, "measurement_kind": kind, "execution_kind": audit["execution_kind"],
                "precision_verified": bool(metadata.get("tensor_precision_probe"))
                if key in ("fp32", "fp64", "tf32") else audit["instruction_precision_verified"],
                "accumulator_dtype": accumulator, "output_dtype": accumulator,
                "blocks": blocks, "iterations": args.iterations, **rate, **descriptor,
                "input_pattern": input_pattern(key, args.inputs),
                "accumulation_policy": accumulation_policy(key, args),
                "precision_probe": metadata.get("tensor_precision_probe"),
                "correctness": correctness, "compiled": audit,
                "kernel": config["kernel"], "status": "ok", **timing,
            }
            rows.append(row)
            print(f"  {config['kernel']:8s} {m:4d}/{n}/{k:<4d} {config['chains']:5d} "
                  f"{blocks_per_sm:9d} {timing['median_ms']:11.4f} {timing['min_ms']:8.4f} "
                  f"{rate['median_teraops_per_second']:12.2f} {rate['peak_teraops_per_second']:10.2f}"
                  f" {info['registers_per_thread']:5d}", flush=True)
            del a, b, c, extras
    successful = [row for row in rows if row["status"] == "ok"]
    if not successful:
        emit_tensor_results(metadata, args, rows)
        return
    best = max(successful, key=lambda row: row["peak_teraops_per_second"])
    print(f"Measured {'tensor' if best['compiled']['native_tensor_verified'] else 'SIMT matrix'} "
          f"peak: {best['peak_teraops_per_second']:.2f} {unit} (same configuration median "
          f"{best['median_teraops_per_second']:.2f} {unit}; {best['kernel']} "
          f"{best['config']['block_m']}x{best['config']['block_n']}x{best['config']['block_k']})")
    emit_tensor_results(metadata, args, rows)


def input_pattern(key: str, inputs: str) -> str:
    if inputs == "baseline":
        return ("random E2M1 codes over all 16 values, packed two per uint8; unit E8M0 scales"
                if key == "fp4" else "random integers in [-3, 3]" if key == "int8"
                else "random integers in [-3, 3] / 4")
    return ("random one-hot A; random signed B; dense MMA operations" if key == "fp8"
            else "random ternary integers" if key == "int8"
            else "random E2M1 codes for +/-0.5 and +/-1.0, packed two per uint8; unit E8M0 scales"
            if key == "fp4" else "random ternary exact binary fractions")


def accumulation_policy(key: str, args) -> str:
    return {"fp8": "tensor-core FP8 products with FP32 accumulation in tensor memory",
            "fp4": "MX E2M1 multiply with E8M0 group scaling and FP32 accumulation",
            "tf32": "TF32 multiply with FP32 accumulation",
            "fp32": "IEEE FP32 multiply and accumulation",
            "int8": "exact INT32 accumulation (no overflow)",
            "fp64": "FP64 multiply and accumulation"}.get(key, "FP32 tensor accumulation")


def emit_tensor_results(metadata, args, rows) -> None:
    successful = any(row.get("status") == "ok" for row in rows)
    unsupported = any(row.get("status") == "unsupported" for row in rows)
    status = "ok" if successful else "unsupported" if unsupported else "error"
    reason = None if successful else "; ".join(dict.fromkeys(
        row.get("reason", "No usable configuration") for row in rows))
    if status == "unsupported":
        emit_unsupported("tensor", metadata, args, reason, details=rows)
    elif status == "error":
        raise RuntimeError(reason or "No usable configuration")
    else:
        emit_results("tensor", metadata, args, rows)


# ---------------------------------------------------------------- GEMM mode
GEMM_KEYS = ("bf16", "fp16", "tf32", "fp32", "fp64", "int8", "fp8", "fp4")
# The reference's GEMM tolerances (bench_tensor.py:289-299); the formats it does
# not run in GEMM mode (fp8, fp4) use exact operands.
GEMM_TOLERANCE = {"bf16": 2e-3, "fp16": 2e-3, "tf32": 1e-2, "fp32": 2e-3, "fp64": 1e-10,
                  "int8": 0.0, "fp8": 0.0, "fp4": 0.0}
# Kernel shape reported in each GEMM row.
GEMM_CONFIG = {
    "fp32": {"block_m": 128, "block_n": 128, "block_k": 8, "stages": 2, "threads": 256,
             "kernel": "simt fma.rn.f32, 8x8 register tile"},
    "fp64": {"block_m": 128, "block_n": 128, "block_k": 16, "stages": 3, "threads": 256,
             "kernel": "mma.sync m16n8k4 f64, cp.async ring"},
}


# K elements per 16-byte unit: the tcgen05 GEMM's TMA rows are whole 16-byte
# units (MX FP4 also whole 32-element scale groups); CUDA-core kinds take any K.
GEMM_K_UNIT = {"bf16": 8, "fp16": 8, "tf32": 4, "int8": 16, "fp8": 16, "fp4": 32,
               "fp32": 1, "fp64": 1}


def gemm_padded_k(key: str, k: int) -> int:
    unit = GEMM_K_UNIT[key]
    return -(-k // unit) * unit


def gemm_inputs(key: str, m: int, n: int, k: int, device, gen):
    """A [M,K'], B [N,K'] (K contiguous) and packed scales for MX FP4.

    bf16/fp16/tf32/fp32/fp64 follow the reference's GEMM inputs
    (bench_tensor.py:249-261): normal A, normal B scaled by 1/sqrt(K); int8 is
    ternary; fp8 uses integers in [-3, 3]/4 and fp4 draws all 16 E2M1 codes with
    unit scales, so those two are exact in FP32.  K' = gemm_padded_k(key, k):
    when K is not a whole number of 16-byte units the rows are zero-padded
    (data preparation outside timing; the padded columns add nothing to C and
    the operation count stays 2*M*N*K).
    """
    kp = gemm_padded_k(key, k)

    def pad(t):
        return t if kp == k else torch.nn.functional.pad(t, (0, kp - k))

    if key == "fp4":
        a_codes = pad(torch.randint(0, 16, (m, k), generator=gen, dtype=torch.uint8))
        b_codes = pad(torch.randint(0, 16, (n, k), generator=gen, dtype=torch.uint8))
        a = pack_e2m1_pairs(a_codes).to(device)
        b = pack_e2m1_pairs(b_codes).to(device)
        sa = torch.full((m, kp // MX_GROUP_SIZE), E8M0_UNIT_SCALE, dtype=torch.uint8, device=device)
        sb = torch.full((n, kp // MX_GROUP_SIZE), E8M0_UNIT_SCALE, dtype=torch.uint8, device=device)
        return a, b, (pack_scales(sa), pack_scales(sb))
    if key == "int8":
        return (pad(torch.randint(-1, 2, (m, k), generator=gen).to(torch.int8)).to(device),
                pad(torch.randint(-1, 2, (n, k), generator=gen).to(torch.int8)).to(device), None)
    if key == "fp8":
        return (pad(torch.randint(-3, 4, (m, k), generator=gen).double() / 4)
                .to(torch.float8_e4m3fn).to(device),
                pad(torch.randint(-3, 4, (n, k), generator=gen).double() / 4)
                .to(torch.float8_e4m3fn).to(device), None)
    dtype = STORAGE[key]
    gen_dtype = torch.float64 if key == "fp64" else torch.float32
    a = pad(torch.randn((m, k), generator=gen, dtype=gen_dtype)).to(dtype).to(device)
    b = pad(torch.randn((n, k), generator=gen, dtype=gen_dtype) * (1.0 / math.sqrt(k))) \
        .to(dtype).to(device)
    return a, b, None


def pack_scales(scales: torch.Tensor) -> torch.Tensor:
    """E8M0 scales [rows][K/32] in the GEMM's packed layout (tcb_mx_scales_pack)."""
    packed = torch.empty(_native.mx_scales_packed_bytes(scales.shape[0], scales.shape[1]),
                         dtype=torch.uint8, device=scales.device)
    _native.mx_scales_pack(scales, packed, scales.shape[0], scales.shape[1])
    return packed


def gemm_reference(key: str, a, b) -> torch.Tensor:
    """FP32 (INT32, FP64) reference product on the device, full precision (no TF32)."""
    if key == "fp64":
        return torch.matmul(a, b.t())
    previous = torch.backends.cuda.matmul.fp32_precision
    torch.backends.cuda.matmul.fp32_precision = "ieee"
    try:
        if key == "fp4":
            av, bv = decode_e2m1(a).float(), decode_e2m1(b).float()
        else:
            av, bv = a.float(), b.float()
        out = torch.matmul(av, bv.t())
    finally:
        torch.backends.cuda.matmul.fp32_precision = previous
    return out.to(torch.int32) if key == "int8" else out


def run_gemm(args, metadata) -> None:
    key = math_key(args)
    device = torch.device("cuda", args.device)
    sizes = args.sizes
    unit = "TOPS" if key == "int8" else "TFLOP/s"
    kernel_text = (GEMM_CONFIG[key]["kernel"] if key in GEMM_CONFIG
                   else "tcgen05 persistent 256x256 tiles (128x256 for MX FP4)")
    print(f"\nMatrix GEMM: {key} inputs, {accumulator_name(key).upper()} accumulate/output; "
          f"2*M*N*K operations; {kernel_text}")
    print("     N  median ms  min ms  median " + unit + "  peak " + unit + "  max abs error")
    info = _native.kernel_info(_native.FAMILY_GEMM, NATIVE[key])
    probe = metadata.get("tensor_precision_probe")
    audit = compiled_info(key, info, bool(probe) if key in ("fp32", "tf32", "fp64") else True)
    rows = []
    gen = torch.Generator().manual_seed(args.seed)
    for size in sizes:
        m = n = k = size
        base = {"mode": "gemm", "m": m, "n": n, "k": k, "dtype": key}
        need = size * size * (64 if key != "fp4" else 16)
        free = available_memory_bytes()
        if free is not None and need > free * 0.8:
            raise RuntimeError(f"N={size} needs about {need / 2**30:.1f} GiB of device memory")
        a, b, scales = gemm_inputs(key, m, n, k, device, gen)
        sa, sb = scales if scales is not None else (None, None)
        c = torch.full((m, n), float("nan") if key != "int8" else 0, device=device,
                       dtype=torch.int32 if key == "int8" else
                       torch.float64 if key == "fp64" else torch.float32)
        if key == "int8":
            c.fill_(-2**31)
        status = torch.zeros(1, dtype=torch.int32, device=device)

        kp = gemm_padded_k(key, k)
        if kp != k:
            base["k_padded"] = kp

        def run():
            _native.gemm(NATIVE[key], a, b, c, m, n, kp, scale_a=sa, scale_b=sb, status=status)

        try:
            run()
        except _native.TcbError as exc:
            if exc.is_capability or exc.is_resource:
                rows.append({**base, "status": "unsupported" if exc.is_capability else "skipped",
                             "reason": str(exc)})
                continue
            raise
        torch.cuda.synchronize()
        if int(status.item()) != 0:
            raise RuntimeError(f"device-side wait failed: {_native.strerror(int(status.item()))}")
        reference = gemm_reference(key, a, b)
        tol = GEMM_TOLERANCE[key]
        torch.testing.assert_close(c, reference, rtol=tol, atol=tol)
        max_err = (c.double() - reference.double()).abs().max().item()
        correctness = {"passed": True, "max_abs_error": max_err, "rtol": tol, "atol": tol,
                       "reference": "exact ternary product converted to INT32" if key == "int8"
                       else "FP64 torch.matmul" if key == "fp64"
                       else "FP32 torch.matmul of the decoded operands, IEEE precision"}
        del reference
        timing = measure(run, args)
        rate = rates(2 * m * n * k, timing, key)
        descriptor = precision_descriptor(args.dtype, args.input_precision)
        if key in GEMM_CONFIG:
            config = dict(GEMM_CONFIG[key])
        else:
            # The tile and ring the library runs for this shape, as it reports them.
            shape = _native.kernel_info(_native.FAMILY_GEMM, NATIVE[key], m, n)
            config = {"block_m": shape["tile_m"], "block_n": shape["tile_n"],
                      "block_k_bytes": 128, "stages": shape["pipeline_stages"],
                      "persistent": True, "cta_pair": shape["cluster_ctas"] == 2}
        row = {**base,
               "measurement_kind": (f"{descriptor['math_mode']}_gemm"
                                    if args.dtype in ("fp32", "fp64") else "dense_tensor_gemm"),
               "execution_kind": audit["execution_kind"],
               "precision_verified": bool(probe) if args.dtype in ("fp32", "fp64")
               else audit["instruction_precision_verified"],
               "accumulator_dtype": accumulator_name(key), "output_dtype": accumulator_name(key),
               **descriptor, **rate, "config": config,
               "status": "ok", "correctness": correctness, "precision_probe": probe,
               "compiled": audit, **timing}
        rows.append(row)
        print(f"{size:6d} {timing['median_ms']:10.4f} {timing['min_ms']:7.4f} "
              f"{rate['median_teraops_per_second']:12.2f} {rate['peak_teraops_per_second']:10.2f} "
              f"{max_err:.3g}", flush=True)
        del a, b, c, scales
        torch.cuda.empty_cache()
    emit_tensor_results(metadata, args, rows)


def build_parser():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--mode", choices=("peak", "gemm"), default="peak",
                        help="resident matrix-compute peak (default), or application-style GEMM")
    parser.add_argument("--iterations", type=int, default=1024,
                        help="resident MMA repeats, 1..262144; FP8/FP4 maximum 4096 (default: 1024)")
    parser.add_argument("--blocks-per-sm", nargs="+", type=int, default=[1, 2, 4, 8],
                        help="launched CTAs per SM (default: 1 2 4 8)")
    parser.add_argument("--sizes", nargs="+", type=int, default=[2048, 4096, 8192],
                        help="square GEMM dimensions M=N=K (default: 2048 4096 8192)")
    parser.add_argument("--dtype", choices=("fp16", "bf16", "fp8", "fp4", "fp32", "tf32", "int8",
                                            "fp64"), default="fp16")
    parser.add_argument("--input-precision", choices=("ieee", "tf32"),
                        help="math mode for --dtype fp32 (default: ieee)")
    parser.add_argument("--inputs", choices=("reference", "baseline"), default="reference",
                        help="operand set: the reference suite's, or integers in [-3,3] "
                             "with one chain")
    parser.add_argument("--tiles", nargs="+",
                        help="restrict the sweep to tiles given as MxN or MxNxK")
    parser.add_argument("--block-k", type=int, help="override tile K of every candidate")
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--quick", action="store_true",
                        help="smoke test: one tile and 64 repeats")
    add_common_arguments(parser)
    return parser


def main(argv=None) -> None:
    parser = build_parser()
    args = parser.parse_args(argv)
    normalize_precision_args(parser, args)
    if not 1 <= args.iterations <= 262144:
        parser.error("--iterations must be between 1 and 262144 for exact FP32 validation")
    if any(v <= 0 for v in args.blocks_per_sm):
        parser.error("--blocks-per-sm values must be positive")
    if args.dtype in ("fp8", "fp4") and args.iterations > 4096:
        parser.error("FP8/FP4 peak limits --iterations to 4096 for exact FP32 accumulation")
    metadata = setup_device(args)
    metadata.update(precision_descriptor(args.dtype, args.input_precision))
    if args.mode == "gemm":
        key = math_key(args)
        if key not in GEMM_KEYS:
            emit_not_implemented("tensor", metadata, args,
                                 f"This build's GEMM mode covers {', '.join(sorted(GEMM_KEYS))}; "
                                 f"{key} GEMM is not implemented")
            return
        if key in ("fp32", "tf32", "fp64"):
            try:
                metadata["tensor_precision_probe"] = validate_gemm_precision(
                    torch.device("cuda", args.device), key)
            except TensorUnsupportedError as exc:
                emit_unsupported("tensor", metadata, args, str(exc))
                return
        run_gemm(args, metadata)
        return
    if not metadata["architecture"].startswith("sm_10"):
        emit_unsupported("tensor", metadata, args,
                         f"libtcb targets sm_100a; device is {metadata['architecture']}")
        return
    device = torch.device("cuda", args.device)
    torch.manual_seed(0)
    try:
        if args.dtype == "fp32":
            metadata["tensor_precision_probe"] = validate_fp32_precision(device,
                                                                         args.input_precision)
        elif args.dtype == "fp64":
            metadata["tensor_precision_probe"] = validate_fp64_precision(device, _native.TV_DMMA)
            metadata["tensor_precision_probe_simt"] = validate_fp64_precision(device,
                                                                              _native.TV_SIMT)
        elif args.dtype == "fp8":
            metadata["tensor_storage_probe"] = validate_fp8_storage(device)
        elif args.dtype == "fp4":
            metadata["tensor_dot_lowering_probe"] = validate_fp4_arithmetic(device)
    except TensorUnsupportedError as exc:
        emit_unsupported("tensor", metadata, args, str(exc))
        return
    except _native.TcbError as exc:
        if exc.is_capability:
            emit_unsupported("tensor", metadata, args, str(exc))
            return
        raise
    run_peak(args, metadata)


if __name__ == "__main__":
    main()
