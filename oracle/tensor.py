"""Resident tensor-probe oracle (numpy) - test infrastructure.

Restates, from the reference suite's bench_tensor.py:
  E2M1_VALUES / E8M0 constants       bench_tensor.py:55-69
  pack_e2m1_pairs                    bench_tensor.py:603-611
  peak_tolerance                     bench_tensor.py:302-325
  validate_peak (accept / reject)    bench_tensor.py:328-346
  resident_reference (A.B * iters)   bench_tensor.py:277-286, 1231-1232
  fp4 decode + scale                 bench_tensor.py:614-644, 829-886 (OCP MX v1.0)
  fp32 / fp64 precision probes       bench_tensor.py:675-757
All arithmetic is exact: FP64 for binary fractions, int64 for INT8.
"""

from __future__ import annotations

import numpy as np

FP4_PACKING_FACTOR = 2
MX_GROUP_SIZE = 32
E8M0_UNIT_SCALE = 127
_E2M1_MAGNITUDES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E2M1_VALUES = _E2M1_MAGNITUDES + tuple(-v for v in _E2M1_MAGNITUDES)


def pack_e2m1_pairs(codes: np.ndarray) -> np.ndarray:
    """Two 4-bit codes per byte along the last axis; even index -> low nibble."""
    codes = np.asarray(codes, dtype=np.uint16)
    return ((codes[..., 1::2] << 4) | codes[..., 0::2]).astype(np.uint8)


def unpack_e2m1(packed: np.ndarray) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = packed & 0xF
    out[..., 1::2] = packed >> 4
    return out


def decode_e2m1(packed: np.ndarray) -> np.ndarray:
    return np.asarray(E2M1_VALUES, dtype=np.float64)[unpack_e2m1(packed)]


def e8m0_value(code: int) -> float:
    """E8M0 scale: 2**(code - 127); code 255 is NaN."""
    return float("nan") if code == 255 else 2.0 ** (int(code) - 127)


def pack_mx_scales(scales: np.ndarray) -> np.ndarray:
    """The GEMM's packed E8M0 layout (this build's own format, flat uint8).

    Rows are padded to a multiple of 256 and groups to a multiple of 8 with the
    unit scale 127; then, per 128 rows and 8 groups, a 1 KB block of two
    512-byte halves (groups 0-3, 4-7) in which lane l = r % 32 holds the four
    groups of rows l, 32+l, 64+l, 96+l:
    out[((r//128)*(groups_p//8) + g//8)*1024 + (g%8//4)*512 + (r%32)*16
        + (r%128//32)*4 + g%4] = scales[r, g].
    """
    rows, groups = scales.shape
    rows_p, groups_p = -(-rows // 256) * 256, -(-groups // 8) * 8
    padded = np.full((rows_p, groups_p), E8M0_UNIT_SCALE, dtype=np.uint8)
    padded[:rows, :groups] = scales
    # axes: row block, row quarter j, lane l, group block, half h, group b
    s = padded.reshape(rows_p // 128, 4, 32, groups_p // 8, 2, 4)
    return np.ascontiguousarray(s.transpose(0, 3, 4, 2, 1, 5)).reshape(-1)


def peak_tolerance(dtype: str, block_k: int, iterations: int) -> float:
    if dtype == "int8":
        return 0.0
    if dtype == "fp4":
        return 4.0 * iterations * block_k * 2.0**-24
    unit = 2.0**-53 if dtype == "fp64" else 2.0**-24
    return 4.0 * iterations * block_k * (1.0 / 256.0) * unit


def validate_peak(c: np.ndarray, reference: np.ndarray, dtype: str, block_k: int,
                  iterations: int) -> bool:
    """True when every |c - reference| <= tolerance (rtol 0), NaN rejected."""
    c = np.asarray(c, dtype=np.float64)
    reference = np.asarray(reference, dtype=np.float64)
    if c.shape != reference.shape:
        return False
    err = np.abs(c - reference)
    return bool(np.all(err <= peak_tolerance(dtype, block_k, iterations)))


def resident_reference(a: np.ndarray, b_nk: np.ndarray, iterations: int, dtype: str,
                       scale_a: np.ndarray | None = None,
                       scale_b: np.ndarray | None = None) -> np.ndarray:
    """iterations * (A . B^T) for A [..., M, K] and B stored as [..., N, K].

    dtype fp4: A and B are packed E2M1 bytes, scales [.., rows, K/32] E8M0.
    The result is float64 (int64 for int8); exact for the probes' operands.
    """
    if dtype == "fp4":
        av = decode_e2m1(a)
        bv = decode_e2m1(b_nk)
        if scale_a is not None:
            av = av * np.repeat(2.0 ** (scale_a.astype(np.float64) - 127), MX_GROUP_SIZE, axis=-1)
        if scale_b is not None:
            bv = bv * np.repeat(2.0 ** (scale_b.astype(np.float64) - 127), MX_GROUP_SIZE, axis=-1)
        return np.matmul(av, np.swapaxes(bv, -1, -2)) * iterations
    if dtype == "int8":
        prod = np.matmul(a.astype(np.int64), np.swapaxes(b_nk.astype(np.int64), -1, -2))
        return prod * iterations
    prod = np.matmul(a.astype(np.float64), np.swapaxes(b_nk.astype(np.float64), -1, -2))
    return prod * iterations


def fp32_probe_expected(precision: str, m: int, n: int, k: int) -> tuple[np.ndarray, np.ndarray]:
    """(A, expected C) of the IEEE/TF32 probe with B = identity [n, k]."""
    tail, mantissa, exponent = 1.0 + 2.0**-12, 1.0 + 2.0**-9, 2.0**20
    a = np.full((m, k), tail, dtype=np.float32)
    a[0, 1], a[0, 2] = mantissa, exponent
    expected = np.zeros((m, n), dtype=np.float32)
    expected[:, :k] = a if precision == "ieee" else 1.0
    if precision == "tf32":
        expected[0, 1], expected[0, 2] = mantissa, exponent
    return a, expected


def fp64_probe_expected(m: int, n: int, k: int) -> tuple[np.ndarray, np.ndarray]:
    a = np.full((m, k), 1.0 + 2.0**-40, dtype=np.float64)
    a[:, 0] = np.arange(1, m + 1, dtype=np.float64)
    expected = np.zeros((m, n), dtype=np.float64)
    expected[:, :k] = a
    return a, expected


def tf32_truncate(x: np.ndarray) -> np.ndarray:
    """FP32 values with the 13 low mantissa bits cleared (TF32 operand view)."""
    bits = np.asarray(x, dtype=np.float32).view(np.uint32) & np.uint32(0xFFFFE000)
    return bits.view(np.float32)
