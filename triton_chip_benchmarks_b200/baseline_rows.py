"""The north-star configurations as validated, clock-stamped rows (one GPU).

bench.py times the headline copy; this module measures, outside that timed
region, one row per configuration of the benchmark's own table, on the same
GPU and through the same library:

* ``tensor_<dtype>``: the resident probe with the baseline operand set
  (integers in [-3, 3], scaled by 1/4 for the float formats; MX FP4 drawn
  over all 16 E2M1 codes with unit E8M0 scales), one CTA per SM, 4096
  reissues, K = 64 (bf16, fp16), 32 (tf32, fp32, fp64), 128 (int8, fp8) or
  256 (MX FP4), tiles 128 x 256 and 256 x 256 swept on the tensor cores;
* ``vector_<dtype>``: 4 x SMs CTAs x 256 threads, 8 accumulator registers
  per thread, 8192 iterations of x = x * (1 - 2**-10) + 2**-10 from
  x0 ~ U[0.5, 1) (int8 row: int32 x = x * 1 + 1 with wrap-around);
* ``gemm_fp4``: the MX FP4 GEMM at M = N = K = 8192, unit scales, fp32 C.

Each configuration is validated on its first launch (tensor rows and the GEMM
exactly against the product computed on the device in float64; chains bit for
bit against a single-rounding replay, fp64 by the closed form), then timed:
W untimed launches and K timed launches, each between its own CUDA events on
the launching stream.  ``value`` is the fastest launch (the reference's peak
convention) and ``median`` the median launch.  The SM clock is sampled during
the timed launches, so every row also gives the median launch's fraction of
the ceiling at the median clock (per-SM rate x SMs x clock): a row below the
datasheet but near that ceiling is limited by the clock the power cap allows,
not by the kernel.  The GEMM flushes L2 between launches (its 64 MiB of operands
would otherwise stay cached); the probes keep their operands on chip by
design, so L2 plays no part in them.
"""

from __future__ import annotations

import math
import statistics
from types import SimpleNamespace

import torch

from . import _native, bench_tensor, bench_vector
from .clocks import ClockSampler
from .validation import validate_relative

TENSOR_ITERATIONS = 4096
VECTOR_ITERATIONS = 8192

# HGX B200 dense datasheet figures per GPU (TFLOP/s or TOP/s).  The B200
# datasheet gives no non-tensor FP16/BF16 or INT32 rate; those rows use the
# derived ceiling at the maximum clock and say so.
DATASHEET = {"tensor_bf16": 2250.0, "tensor_fp16": 2250.0, "tensor_tf32": 1125.0,
             "tensor_fp32": 75.0, "tensor_fp64": 37.0, "tensor_int8": 4500.0,
             "tensor_fp8": 4500.0, "tensor_fp4": 9000.0, "gemm_fp4": 9000.0,
             "vector_fp32": 75.0, "vector_fp64": 37.0}
# Operations per SM per clock of the unit each row runs on (2 per multiply-add).
PER_SM_CLOCK = {"tensor_bf16": 8192, "tensor_fp16": 8192, "tensor_tf32": 4096,
                "tensor_fp32": 256, "tensor_fp64": 128, "tensor_int8": 16384,
                "tensor_fp8": 16384, "tensor_fp4": 32768, "gemm_fp4": 32768,
                "vector_bf16": 256, "vector_fp16": 256, "vector_fp32": 256,
                "vector_fp64": 128, "vector_int8": 128}

# key: (variant, K, tiles)
TENSOR_CONFIGS = {
    "bf16": (_native.TV_TCGEN05, 64, ((128, 256), (256, 256))),
    "fp16": (_native.TV_TCGEN05, 64, ((128, 256), (256, 256))),
    "tf32": (_native.TV_TCGEN05, 32, ((128, 256), (256, 256))),
    "fp32": (_native.TV_SIMT_REG, 32, ((256, 256),)),
    "fp64": (_native.TV_DMMA, 32, ((256, 256),)),
    "int8": (_native.TV_TCGEN05, 128, ((128, 256), (256, 256))),
    "fp8": (_native.TV_TCGEN05, 128, ((128, 256), (256, 256))),
    "fp4": (_native.TV_TCGEN05, 256, ((128, 256), (256, 256))),
}
# key: (native dtype, elements per thread, unroll); the packed 16-bit formats
# hold two elements per accumulator register.
VECTOR_CONFIGS = {
    "bf16": (_native.V_BF16, 2, 16), "fp16": (_native.V_FP16, 2, 16),
    "fp32": (_native.V_FP32, 1, 16), "fp64": (_native.V_FP64, 1, 16),
    "int8": (_native.V_INT32_IMAD, 1, 16),
}


def _launch_count(single_ms: float, window_ms: float) -> int:
    return max(5, min(400, math.ceil(window_ms / max(single_ms, 1e-3))))


def _time_launches(run, device_index: int, warmup: int, window_ms: float, between=None) -> dict:
    """Per-launch CUDA-event times of `run` on the current stream, with clocks."""
    stream = torch.cuda.current_stream()
    probe = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    probe[0].record(stream)
    run()
    probe[1].record(stream)
    torch.cuda.synchronize()
    count = _launch_count(probe[0].elapsed_time(probe[1]), window_ms)
    for _ in range(warmup):
        if between is not None:
            between()
        run()
    torch.cuda.synchronize()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(count)]
    with ClockSampler(device_index) as sampler:
        for start, end in events:
            if between is not None:
                between()
            start.record(stream)
            run()
            end.record(stream)
        torch.cuda.synchronize()
    times = [start.elapsed_time(end) for start, end in events]
    return {"min_ms": min(times), "median_ms": statistics.median(times), "launches": count,
            "warmup": warmup, "clocks": sampler.summary()}


def _row(name: str, ops: int, timing: dict, config: dict, validation: dict, sms: int,
         peaks: dict) -> dict:
    unit = "TOP/s" if name.endswith("int8") else "TFLOP/s"
    value = ops / (timing["min_ms"] * 1e-3) / 1e12
    median = ops / (timing["median_ms"] * 1e-3) / 1e12
    row = {"status": "ok", "value": value, "median": median, "unit": unit,
           "operations_per_launch": ops, "config": config, "validation": validation,
           "timing": {k: timing[k] for k in ("min_ms", "median_ms", "launches", "warmup")},
           "clocks": timing["clocks"]}
    if name in DATASHEET:
        row["datasheet"] = DATASHEET[name]
        row["frac_datasheet"] = value / DATASHEET[name]
    mhz = timing["clocks"].get("sm_mhz")
    max_mhz = timing["clocks"].get("sm_max_mhz")
    if name not in DATASHEET and max_mhz:
        row["datasheet"] = PER_SM_CLOCK[name] * sms * max_mhz * 1e6 / 1e12
        row["datasheet_note"] = "derived: per-SM rate x SMs x maximum clock (no datasheet figure)"
        row["frac_datasheet"] = value / row["datasheet"]
    if mhz:
        # Median launch against the median sampled clock (the fastest launch
        # may have run above the median clock).
        ceiling = PER_SM_CLOCK[name] * sms * mhz * 1e6 / 1e12
        row["ceiling_at_sampled_clock"] = ceiling
        row["frac_ceiling_at_sampled_clock"] = median / ceiling
    if name == "tensor_bf16" and peaks.get("bf16_tflops_sustained"):
        row["frac_measured_bf16_sustained"] = value / peaks["bf16_tflops_sustained"]
    return row


def tensor_row(key: str, device: torch.device, sms: int, warmup: int, window_ms: float,
               peaks: dict, seed: int = 0) -> dict:
    variant, k, tiles = TENSOR_CONFIGS[key]
    name = f"tensor_{key}"
    best = None
    for m, n in tiles:
        config = {"block_m": m, "block_n": n, "block_k": k, "chains": 1, "variant": variant,
                  "kernel": bench_tensor.VARIANT_NAMES[variant]}
        gen = torch.Generator().manual_seed(seed)
        for _ in range(8):
            a, b, c, extras = bench_tensor.peak_inputs(key, "baseline", sms, config, device, gen)
            # MX FP4 over all 16 codes: 4096 x S is exact in fp32 only while max|S| < 1024.
            if key != "fp4" or bench_tensor.fp4_exactness(a, b, TENSOR_ITERATIONS) < 1024:
                break
        else:
            raise RuntimeError("no FP4 operand draw kept 4096 x S exact in fp32")
        status = torch.zeros(1, dtype=torch.int32, device=device)

        def run():
            bench_tensor.launch(key, config, a, b, c, extras, sms, 1, TENSOR_ITERATIONS, status)

        c.fill_(-2**31 if key == "int8" else float("nan"))
        run()
        torch.cuda.synchronize()
        if int(status.item()) != 0:
            raise RuntimeError(f"device-side wait failed: {_native.strerror(int(status.item()))}")
        reference = bench_tensor.reference_output(key, a, b, extras, TENSOR_ITERATIONS)
        validation = validate_relative(c, reference, bench_tensor.BASELINE_RTOL[key])
        validation["reference"] = "float64 product on the device x 4096"
        del reference
        timing = _time_launches(run, device.index or 0, warmup, window_ms)
        if int(status.item()) != 0:
            raise RuntimeError(f"device-side wait failed: {_native.strerror(int(status.item()))}")
        ops = 2 * m * n * k * TENSOR_ITERATIONS * sms
        row = _row(name, ops, timing, {**config, "blocks": sms, "blocks_per_sm": 1,
                                       "iterations": TENSOR_ITERATIONS,
                                       "operands": bench_tensor.input_pattern(key, "baseline")},
                   validation, sms, peaks)
        if best is None or row["value"] > best["value"]:
            best = row
        del a, b, c, extras
    return best


def vector_row(key: str, device: torch.device, sms: int, warmup: int, window_ms: float,
               peaks: dict, seed: int = 0) -> dict:
    code, ept, unroll = VECTOR_CONFIGS[key]
    blocks, threads = 4 * sms, 256
    elements = blocks * threads * ept
    args = SimpleNamespace(dtype=key, inputs="baseline", int8_op="imad", seed=seed)
    inputs, coeff = bench_vector.make_inputs(args, elements, device)
    coeff_arg = _native.vector_coefficients(code, coeff, coeff.cpu().contiguous())
    output = torch.empty_like(inputs)

    def run():
        _native.vector_chains(code, inputs, output, coeff_arg, elements, VECTOR_ITERATIONS,
                              blocks, threads, ept, unroll)

    run()
    torch.cuda.synchronize()
    validation = bench_vector.validate(args, inputs, output, coeff, VECTOR_ITERATIONS)
    timing = _time_launches(run, device.index or 0, warmup, window_ms)
    ops = 2 * 8 * elements * VECTOR_ITERATIONS
    config = {"blocks": blocks, "threads": threads, "elements_per_thread": ept,
              "accumulator_registers_per_thread": 8, "unroll": unroll,
              "coefficients": "registers" if code in _native.COEFF_IN_REGISTERS else "by value",
              "iterations": VECTOR_ITERATIONS,
              "operation": "int32 x*1+1 (wrap)" if key == "int8" else "x*a+b, a=1-2^-10, b=2^-10"}
    return _row(f"vector_{key}", ops, timing, config, validation, sms, peaks)


def gemm_fp4_row(device: torch.device, sms: int, warmup: int, window_ms: float, peaks: dict,
                 size: int = 8192, seed: int = 0) -> dict:
    gen = torch.Generator().manual_seed(seed)
    a, b, (sa, sb) = bench_tensor.gemm_inputs("fp4", size, size, size, device, gen)
    c = torch.full((size, size), float("nan"), device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)  # 2 x the 126 MB L2

    def run():
        _native.gemm(_native.T_MXF4, a, b, c, size, size, size, scale_a=sa, scale_b=sb,
                     status=status)

    run()
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError(f"device-side wait failed: {_native.strerror(int(status.item()))}")
    reference = bench_tensor.gemm_reference("fp4", a, b)
    if not torch.equal(c, reference):
        raise AssertionError(f"{int((c != reference).sum().item())} GEMM entries differ")
    del reference
    validation = {"passed": True, "exact": True,
                  "reference": "fp32 torch.matmul (IEEE) of the decoded operands on the device"}
    timing = _time_launches(run, device.index or 0, warmup, window_ms,
                            between=lambda: flush.zero_())
    if int(status.item()) != 0:
        raise RuntimeError(f"device-side wait failed: {_native.strerror(int(status.item()))}")
    shape = _native.kernel_info(_native.FAMILY_GEMM, _native.T_MXF4, size, size)
    config = {"m": size, "n": size, "k": size, "scales": "E8M0 127 (unit), one per 32 K",
              "tile_m": shape["tile_m"], "tile_n": shape["tile_n"],
              "cluster_ctas": shape["cluster_ctas"], "stages": shape["pipeline_stages"],
              "l2": "flushed between launches (256 MiB write)"}
    return _row("gemm_fp4", 2 * size ** 3, timing, config, validation, sms, peaks)


def measure_rows(device: torch.device, peaks: dict, warmup: int = 3,
                 window_ms: float = 250.0) -> dict:
    """Every row, in table order; a row that fails records its error and the
    others still run."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    jobs = [(f"tensor_{key}", lambda key=key: tensor_row(key, device, sms, warmup, window_ms,
                                                          peaks))
            for key in TENSOR_CONFIGS]
    jobs += [(f"vector_{key}", lambda key=key: vector_row(key, device, sms, warmup, window_ms,
                                                          peaks))
             for key in VECTOR_CONFIGS]
    jobs.append(("gemm_fp4", lambda: gemm_fp4_row(device, sms, warmup, window_ms, peaks)))
    rows = {}
    for name, job in jobs:
        try:
            rows[name] = job()
        except Exception as exc:  # noqa: BLE001 - recorded in the row, the rest still run
            rows[name] = {"status": "error", "reason": f"{type(exc).__name__}: {exc}"}
        torch.cuda.empty_cache()
    return rows
