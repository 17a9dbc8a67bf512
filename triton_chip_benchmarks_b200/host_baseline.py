"""Host-side baselines: the reference suite's validation paths timed on the CPU.

These are reported baselines, not targets.  Each one is what the reference
computes on the host to check a device result, written with torch on the CPU:

  tile        BASELINE's CPU-runnable case: A[128x64] . B[64x128] bf16 with values
              uniform over {-2, -1.5, ..., 2} / 4, accumulated 4 times into an
              fp32 accumulator, checked against torch.matmul in fp32
              (the reference's _reference, bench_tensor.py:277-286)
  tensor      _reference for one CTA's resident tile (bench_tensor.py:277-286,
              1231-1232): one fp32 (fp64 for fp64) matmul of a 256 x K by K x 256
              tile, scaled by the iteration count
  vector      the host recurrence of check_output (bench_vector.py:322-372) over
              one 131072-element chunk of 8 chains: x <- x * a + b, 256 steps

Rates count the reference's own operations (2 per multiply-add) over the best of
at least five timed repeats (median also reported); `threads` is
torch.get_num_threads() and `cpu_count` os.cpu_count() of the host that ran it.
Run: python -m triton_chip_benchmarks_b200.host_baseline [--output FILE]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import time

import torch

CHUNK = 131072  # elements per chain checked at a time by the reference's check_output
CHAINS = 8


def _timed(fn, repeats: int) -> tuple[float, float]:
    """(best, median) seconds of fn() over `repeats` runs after one warm-up run."""
    fn()
    samples = []
    for _ in range(repeats):
        start = time.perf_counter()
        fn()
        samples.append(time.perf_counter() - start)
    return min(samples), statistics.median(samples)


def tile_baseline(repeats: int = 20, seed: int = 0) -> dict:
    gen = torch.Generator().manual_seed(seed)
    levels = torch.arange(-4, 5, dtype=torch.float32) / 8  # {-2, -1.5, ..., 2} / 4
    a = levels[torch.randint(0, 9, (128, 64), generator=gen)].to(torch.bfloat16)
    b = levels[torch.randint(0, 9, (64, 128), generator=gen)].to(torch.bfloat16)
    reps = 4

    def accumulate():
        acc = torch.zeros(128, 128, dtype=torch.float32)
        af, bf = a.float(), b.float()
        for _ in range(reps):
            acc += af @ bf
        return acc

    result = accumulate()
    expected = torch.matmul(a.float(), b.float()) * reps
    if not torch.equal(result, expected):
        raise AssertionError("tile accumulation differs from the fp32 matmul reference")
    best, median = _timed(accumulate, repeats)
    ops = 2 * 128 * 128 * 64 * reps
    return {"case": "tile", "shape": "A[128x64] . B[64x128] bf16, 4 accumulations in fp32",
            "operations": ops, "best_s": best, "median_s": median,
            "gflops": ops / best / 1e9, "median_gflops": ops / median / 1e9,
            "check": "bit-equal to 4 x torch.matmul(A.float(), B.float())"}


def tensor_baseline(dtype: str, repeats: int = 10, seed: int = 0) -> dict:
    k = {"bf16": 64, "fp16": 64, "tf32": 32, "fp32": 32, "fp64": 32, "int8": 128,
         "fp8": 128}[dtype]
    gen = torch.Generator().manual_seed(seed)
    wide = torch.float64 if dtype == "fp64" else torch.float32
    scale = 1 if dtype == "int8" else 4  # integers in [-3, 3], / 4 for the float kinds
    a = torch.randint(-3, 4, (256, k), generator=gen).to(wide) / scale
    b = torch.randint(-3, 4, (k, 256), generator=gen).to(wide) / scale
    iterations = 4096

    def reference():
        return torch.matmul(a, b) * iterations

    best, median = _timed(reference, repeats)
    ops = 2 * 256 * 256 * k
    return {"case": "tensor", "dtype": dtype, "shape": f"256x{k} . {k}x256 in {wide}, x {iterations}",
            "operations": ops, "best_s": best, "median_s": median,
            "gflops": ops / best / 1e9, "median_gflops": ops / median / 1e9}


def vector_baseline(dtype: str, steps: int = 256, repeats: int = 5, seed: int = 0) -> dict:
    wide = torch.float64 if dtype == "fp64" else torch.float32
    gen = torch.Generator().manual_seed(seed)
    x0 = torch.rand((CHAINS, CHUNK), generator=gen, dtype=torch.float64).to(wide) * 0.5 + 0.5
    a = torch.tensor(0.9990234375, dtype=wide)
    b = torch.full((CHAINS, 1), 0.0009765625, dtype=wide)

    def recurrence():
        x = x0.clone()
        for _ in range(steps):
            x = torch.addcmul(b, x, a)
        return x

    best, median = _timed(recurrence, repeats)
    ops = 2 * CHAINS * CHUNK * steps
    return {"case": "vector", "dtype": dtype, "shape": f"{CHAINS} chains x {CHUNK} elements, "
            f"{steps} steps of x*a+b in {wide}", "operations": ops, "best_s": best,
            "median_s": median, "gflops": ops / best / 1e9, "median_gflops": ops / median / 1e9}


def run_all(quick: bool = False) -> dict:
    repeats = 3 if quick else None
    rows = [tile_baseline(**({"repeats": repeats} if quick else {}))]
    for dtype in ("bf16", "fp32", "fp64", "int8"):
        rows.append(tensor_baseline(dtype, **({"repeats": repeats} if quick else {})))
    for dtype in ("fp32", "fp64"):
        rows.append(vector_baseline(dtype, **({"repeats": repeats, "steps": 8} if quick else {})))
    return {"benchmark": "host_baselines", "cpu_count": os.cpu_count(),
            "threads": torch.get_num_threads(), "torch": torch.__version__, "rows": rows}


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--output", help="write the JSON document here as well")
    parser.add_argument("--quick", action="store_true", help="fewer repeats and steps")
    args = parser.parse_args(argv)
    document = run_all(args.quick)
    text = json.dumps(document, indent=1)
    print(text)
    if args.output:
        with open(args.output, "w") as handle:
            handle.write(text + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
