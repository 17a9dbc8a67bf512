"""Vector-chain oracle (numpy) - test infrastructure.

Restates, from the reference suite's bench_vector.py:
  make_inputs (value sets)            bench_vector.py:1191-1216
  throughput_fields (op counting)     bench_vector.py:1271-1280
  closed_form_check                   bench_vector.py:322-372 (check_output)
  dp4a_reference (binary lifting)     bench_vector.py:375-421 (check_int8_output)
  mod256_reference                    bench_vector.py:424-450 (check_int8_mul_add_output)
Exact step-by-step replays live in tcb_oracle.c (oracle.native.chain).
"""

from __future__ import annotations

import math

import numpy as np

CHAINS = 8


def packed_dp4a_weights() -> int:
    packed = sum((v & 255) << s for v, s in zip((3, -2, 1, -1), (0, 8, 16, 24)))
    return packed - 2**32 if packed >= 2**31 else packed


def ops_per_update(dtype: str, int8_mul_add: bool = False) -> int:
    return 8 if dtype == "int8" and not int8_mul_add else 2


def counted_operations(dtype: str, elements: int, iterations: int,
                       int8_mul_add: bool = False) -> int:
    return ops_per_update(dtype, int8_mul_add) * CHAINS * elements * iterations


def closed_form_reference(initial: np.ndarray, coeff: np.ndarray, iterations: int):
    """(reference, tolerance) of x <- a*x + b_c (0 < a < 1 or a == -1), FP64."""
    coeff = np.asarray(coeff, dtype=np.float64)
    a = coeff[0]
    b = coeff[1:, None]
    x0 = np.asarray(initial, dtype=np.float64)
    if a == -1.0:
        ref = b - x0 if iterations % 2 else x0.copy()
        return ref, np.zeros_like(ref)
    decay = math.exp(iterations * math.log(a))
    geometric = -math.expm1(iterations * math.log(a)) / (1.0 - a)
    ref = decay * x0 + b * geometric
    magnitude = np.maximum(np.abs(x0), np.abs(b / (1.0 - a)))
    return ref, magnitude * geometric  # unit-less; caller scales by factor * u


def closed_form_check(initial, output, coeff, iterations, state_dtype: str,
                      single_rounding: bool = True) -> bool:
    ref, scale = closed_form_reference(initial, coeff, iterations)
    if np.all(scale == 0):
        return bool(np.array_equal(np.asarray(output, dtype=np.float64), ref))
    unit = 2.0**-53 if state_dtype == "fp64" else 2.0**-24
    factor = 2.0 if single_rounding else 4.0
    tol = factor * unit * scale + 16 * unit
    err = np.abs(np.asarray(output, dtype=np.float64) - ref)
    return bool(np.all(err <= tol))


def _signed_bytes(word: int) -> list[int]:
    out = []
    for shift in (0, 8, 16, 24):
        byte = (int(word) >> shift) & 255
        out.append(byte - 256 if byte >= 128 else byte)
    return out


def dot4(words: np.ndarray, weights) -> np.ndarray:
    words = np.asarray(words, dtype=np.int64)
    out = np.zeros_like(words)
    for shift, weight in zip((0, 8, 16, 24), weights):
        lane = (words >> shift) & 255
        lane = np.where(lane >= 128, lane - 256, lane)
        out += lane * weight
    return out


def dp4a_reference(initial: np.ndarray, coeff: np.ndarray, iterations: int) -> np.ndarray:
    """Exact int32 DP4A chains via a bounded transition table and binary lifting."""
    coeff = np.asarray(coeff, dtype=np.int64)
    weights = _signed_bytes(int(coeff[0]))
    bias = coeff[1:, None]
    bound = 128 * sum(abs(w) for w in weights) + int(np.abs(bias).max())
    states = np.broadcast_to(np.arange(-bound, bound + 1), (CHAINS, 2 * bound + 1))
    step = dot4(states, weights) + bias + bound
    composed = np.broadcast_to(np.arange(2 * bound + 1), (CHAINS, 2 * bound + 1)).copy()
    remaining = iterations - 1
    while remaining:
        if remaining & 1:
            composed = np.take_along_axis(step, composed, axis=1)
        remaining >>= 1
        if remaining:
            step = np.take_along_axis(step, step, axis=1)
    first = dot4(initial, weights) + bias
    return np.take_along_axis(composed, first + bound, axis=1) - bound


def affine_power(multiplier: int, bias: np.ndarray, iterations: int, modulus: int):
    m, c = 1, np.zeros_like(bias, dtype=object)
    step_m, step_c = multiplier % modulus, bias.astype(object) % modulus
    n = iterations
    while n:
        if n & 1:
            c = (step_m * c + step_c) % modulus
            m = (step_m * m) % modulus
        step_c = (step_m * step_c + step_c) % modulus
        step_m = (step_m * step_m) % modulus
        n >>= 1
    return m, c


def mod256_reference(initial: np.ndarray, coeff: np.ndarray, iterations: int) -> np.ndarray:
    coeff = np.asarray(coeff, dtype=np.int64)
    m, c = affine_power(int(coeff[0]), coeff[1:, None], iterations, 256)
    x = np.asarray(initial, dtype=np.int64).astype(object)
    return ((m * x + c + 128) % 256 - 128).astype(np.int64)


def imad_reference(initial: np.ndarray, coeff: np.ndarray, iterations: int) -> np.ndarray:
    coeff = np.asarray(coeff, dtype=np.int64)
    m, c = affine_power(int(coeff[0]), coeff[1:, None], iterations, 2**32)
    x = np.asarray(initial, dtype=np.int64).astype(object) % 2**32
    v = (m * x + c) % 2**32
    return np.where(v >= 2**31, v - 2**32, v).astype(np.int64)
