"""Output validation for the probes (run by the drivers, outside timing).

These are the suite's acceptance checks, stated in PyTorch so they run on the
device (or the host for integer state), one function per check of the
reference suite:

* :func:`peak_tolerance` / :func:`validate_peak` - resident tensor probe
  (bench_tensor.py:302-346);
* :func:`check_output`, :func:`check_int8_output`,
  :func:`check_int8_mul_add_output` - vector chains (bench_vector.py:322-450);
* :func:`check_chain_exact` - per-step single-rounding replay of a float
  chain, used for operand sets the closed form does not cover exactly;
* :func:`check_imad_output` - int32 wrap-around affine chains;
* :func:`check_read` - per-block read sums (bench_bandwidth.py:81-110).
"""

from __future__ import annotations

import math

import torch

CHAINS = 8
CHUNK = 131072

# OCP MX FP4: E2M1 elements, two per byte (low nibble = even K index), one
# E8M0 scale per 32 elements along K; code 127 encodes 2**0.
FP4_PACKING_FACTOR = 2
MX_GROUP_SIZE = 32
E8M0_UNIT_SCALE = 127
E2M1_MAGNITUDES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E2M1_VALUES = E2M1_MAGNITUDES + tuple(-v for v in E2M1_MAGNITUDES)


# ------------------------------------------------------------------- tensor
def accumulator_name(dtype: str) -> str:
    return "int32" if dtype == "int8" else "fp64" if dtype == "fp64" else "fp32"


def peak_tolerance(dtype: str, block_k: int, iterations: int) -> float:
    """Absolute bound on the accumulated rounding of the resident recurrence.

    Operands are multiples of 1/16, so an exact dot entry is a multiple of
    1/256 bounded by block_k/256; the accumulator rounds once per dot, adding
    at most iterations * block_k/256 * u; a factor 4 of headroom stays far
    below the 1/256 step a skipped or merged iteration would cause.  INT8 is
    exact; MX FP4 entries are bounded by block_k itself.
    """
    if dtype == "int8":
        return 0.0
    if dtype == "fp4":
        return 4.0 * iterations * block_k * 2.0**-24
    unit = 2.0**-53 if dtype == "fp64" else 2.0**-24
    return 4.0 * iterations * block_k * (1.0 / 256.0) * unit


def validate_peak(c: torch.Tensor, reference: torch.Tensor, dtype: str, block_k: int,
                  iterations: int) -> dict:
    tolerance = peak_tolerance(dtype, block_k, iterations)
    torch.testing.assert_close(c, reference, rtol=0, atol=tolerance)
    error = (c.double() - reference.double()).abs().max().item()
    return {"passed": True, "max_abs_error": error, "rtol": 0, "atol": tolerance,
            "reference": f"exact {accumulator_name(dtype).upper()} dot * iterations",
            "tolerance_basis": ("exact INT32 equality" if dtype == "int8" else
                                "accumulated accumulator unit roundoff over all iterations, "
                                "far below the 1/256 exact-operand lattice step")}


def validate_relative(c: torch.Tensor, reference: torch.Tensor, rtol: float) -> dict:
    """Element-wise |c - ref| <= rtol * max(|ref|, tiny) (used for the 256x256 tile sets)."""
    ref = reference.double()
    err = (c.double() - ref).abs()
    bound = rtol * ref.abs().clamp_min(1e-30)
    if not torch.all(err <= bound).item():
        raise AssertionError(f"relative check failed: max_abs_error={err.max().item():.6g}")
    rel = (err / ref.abs().clamp_min(1e-30)).max().item()
    return {"passed": True, "max_abs_error": err.max().item(), "max_rel_error": rel,
            "rtol": rtol, "exact": bool(err.max().item() == 0.0)}


def reference_product(a: torch.Tensor, b_nk: torch.Tensor) -> torch.Tensor:
    """A . B for A [..., M, K] and B stored K-contiguous as [..., N, K].

    FP64 operands multiply in FP64; INT8 in FP64 then converted to INT32
    (exact: every partial sum is an integer below 2**53); other formats in
    FP64 then rounded to FP32 (operands are exact binary fractions, so the
    product is exact and the rounding is the only step).
    """
    if a.dtype == torch.int8:
        return torch.matmul(a.double(), b_nk.double().transpose(-1, -2)).to(torch.int32)
    product = torch.matmul(a.double(), b_nk.double().transpose(-1, -2))
    return product if a.dtype == torch.float64 else product.float()


def pack_e2m1_pairs(codes: torch.Tensor) -> torch.Tensor:
    """Pack E2M1 codes two per byte along the last axis (even index -> low nibble)."""
    low = codes[..., 0::2].to(torch.int16)
    high = codes[..., 1::2].to(torch.int16)
    return ((high << 4) | low).to(torch.uint8)


def decode_e2m1(packed: torch.Tensor) -> torch.Tensor:
    """FP64 values of packed E2M1 bytes, unpacked along the last axis."""
    lookup = torch.tensor(E2M1_VALUES, dtype=torch.float64, device=packed.device)
    low = (packed & 0xF).long()
    high = (packed >> 4).long()
    out = torch.stack((lookup[low], lookup[high]), dim=-1)
    return out.reshape(*packed.shape[:-1], packed.shape[-1] * 2)


# ------------------------------------------------------------------- vector
def check_output(inputs, output, coefficients, iterations, single_rounding=True) -> dict:
    """Closed-form check of x <- a*x + b_c (bench_vector.py:322-372).

    a == -1 is the exactly representable involution (tolerance 0); otherwise
    0 < a < 1 and the error of each step, bounded by the unit roundoff times
    the state magnitude, sums as a geometric series.
    """
    coeff = coefficients.detach().cpu().double()
    a = coeff[0].item()
    involution = a == -1.0
    decay = None if involution else math.exp(iterations * math.log(a))
    geometric = None if involution else -math.expm1(iterations * math.log(a)) / (1.0 - a)
    device = output.device
    b = coeff[1:, None].to(device)
    max_error = max_tolerance = 0.0
    for start in range(0, output.shape[1], CHUNK):
        initial = inputs[:, start:start + CHUNK].double()
        actual = output[:, start:start + CHUNK].double()
        if involution:
            reference = b - initial if iterations % 2 else initial
            tolerance = torch.zeros_like(reference)
        else:
            reference = decay * initial + b * geometric
            magnitude = torch.maximum(initial.abs(), (b / (1.0 - a)).abs())
            unit = 2.0**(-53 if inputs.dtype == torch.float64 else -24)
            factor = 2.0 if single_rounding else 4.0
            tolerance = factor * unit * magnitude * geometric + 16 * unit
        error = (actual - reference).abs()
        if not torch.all(error <= tolerance).item():
            raise RuntimeError("Vector correctness failed: non-finite or inaccurate output; "
                               f"max_abs_error={error.max().item():.6g}, "
                               f"max_tolerance={tolerance.max().item():.6g}")
        max_error = max(max_error, error.max().item())
        max_tolerance = max(max_tolerance, tolerance.max().item())
    return {"correctness": "all elements passed analytic FP64 reference and finite check",
            "max_abs_error": max_error, "max_abs_tolerance": max_tolerance,
            "reference_device": str(device),
            "validation_recurrence": "exact involution" if involution else "contractive affine"}


def _round_to(values: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return values.to(dtype).double()


def check_chain_exact(inputs, output, coefficients, iterations, *, sample=None) -> dict:
    """Replay x <- fma(x, a, b_c) step by step with one rounding per step.

    Each step forms x*a + b exactly in FP64 and rounds once to the state
    dtype (exactness is asserted: the operand spans must fit 53 bits).  FP64
    states use torch.addcmul on FP64, whose result equals fma when the exact
    value fits FP64.  The replay runs on ``sample`` columns (all by default).
    """
    dtype = inputs.dtype
    coeff = coefficients.detach().double().to(output.device)
    a, b = coeff[0], coeff[1:, None]
    cols = slice(None) if sample is None else sample
    x = inputs[:, cols].double()
    exact_fp64 = dtype == torch.float64
    for _ in range(iterations):
        product = x * a
        total = product + b
        if not exact_fp64:
            # Two-sum residual: zero iff the FP64 addition was exact.
            residual = (total - product) - b
            if torch.any(residual != 0).item():
                raise RuntimeError("exact replay needs x*a+b representable in FP64")
            x = _round_to(total, dtype)
        else:
            x = total
    actual = output[:, cols].double()
    mismatches = int((actual != x).sum().item())
    if exact_fp64:
        tol = 2.0**-50 * x.abs().clamp_min(2.0**-30)
        if not torch.all((actual - x).abs() <= tol).item():
            raise RuntimeError("FP64 chain replay mismatch beyond 4 ulp")
    elif mismatches:
        raise RuntimeError(f"single-rounding replay mismatch in {mismatches} elements")
    return {"replayed_elements": int(x.numel() // CHAINS), "bit_exact": mismatches == 0,
            "mismatches": mismatches}


def _signed_bytes(word: int) -> list[int]:
    out = []
    for shift in (0, 8, 16, 24):
        byte = (int(word) >> shift) & 255
        out.append(byte - 256 if byte >= 128 else byte)
    return out


def _dot4(words: torch.Tensor, weights) -> torch.Tensor:
    result = torch.zeros_like(words, dtype=torch.int64)
    for shift, weight in zip((0, 8, 16, 24), weights):
        lane = (words >> shift) & 255
        lane = torch.where(lane >= 128, lane - 256, lane)
        result += lane * weight
    return result


def check_int8_output(inputs, output, coefficients, iterations) -> dict:
    """Exact DP4A chain check by binary lifting (bench_vector.py:390-421).

    After one step the state is bounded by 128*sum|w| + |bias|, so the
    remaining iterations compose a transition table over that bounded range.
    """
    coeff = coefficients.detach().cpu().long()
    weights = _signed_bytes(coeff[0].item())
    bias = coeff[1:, None]
    bound = 128 * sum(abs(w) for w in weights) + int(bias.abs().max())
    states = torch.arange(-bound, bound + 1).expand(CHAINS, -1)
    step = _dot4(states, weights) + bias + bound
    composed = torch.arange(2 * bound + 1).expand(CHAINS, -1)
    remaining = iterations - 1
    while remaining:
        if remaining & 1:
            composed = step.gather(1, composed)
        remaining >>= 1
        if remaining:
            step = step.gather(1, step)
    for start in range(0, inputs.shape[1], CHUNK):
        initial = inputs[:, start:start + CHUNK].cpu().long()
        first = _dot4(initial, weights) + bias
        reference = composed.gather(1, first + bound) - bound
        actual = output[:, start:start + CHUNK].cpu().long()
        if not torch.equal(actual, reference):
            raise RuntimeError("Vector INT8 correctness failed: output differs from exact "
                               "signed INT8 dot4 / INT32 state reference")
    return {"correctness": "all elements passed exact INT64 reference",
            "max_abs_error": 0, "max_abs_tolerance": 0, "reference_device": "cpu",
            "validation_recurrence": "signed INT8 dot4 with INT32 bias/state"}


def _affine_power(multiplier: int, bias: torch.Tensor, iterations: int, modulus: int):
    """(m, c) with f^n(x) = m*x + c (mod modulus) for f(x) = multiplier*x + bias."""
    m, c = 1, torch.zeros_like(bias)
    step_m, step_c = multiplier % modulus, bias % modulus
    n = iterations
    while n:
        if n & 1:
            c = (step_m * c + step_c) % modulus
            m = (step_m * m) % modulus
        step_c = (step_m * step_c + step_c) % modulus
        step_m = (step_m * step_m) % modulus
        n >>= 1
    return m, c


def check_int8_mul_add_output(inputs, output, coefficients, iterations) -> dict:
    """Exact (a*x + b) mod 256 chains (bench_vector.py:424-450)."""
    if any(t.dtype != torch.int8 for t in (inputs, output, coefficients)):
        raise RuntimeError("INT8 multiply-add validation requires INT8 input, output and "
                           "coefficients")
    coeff = coefficients.detach().cpu().long()
    m, c = _affine_power(int(coeff[0]), coeff[1:, None], iterations, 256)
    for start in range(0, inputs.shape[1], CHUNK):
        initial = inputs[:, start:start + CHUNK].cpu().long()
        reference = (m * initial + c + 128) % 256 - 128
        actual = output[:, start:start + CHUNK].cpu().long()
        if not torch.equal(actual, reference):
            raise RuntimeError("Vector INT8 correctness failed: output differs from exact "
                               "modular INT8 multiply-add reference")
    return {"correctness": "all elements passed exact modulo-256 INT64 reference",
            "max_abs_error": 0, "max_abs_tolerance": 0, "reference_device": "cpu",
            "validation_recurrence": "INT8 multiply-add with modulo-256 state"}


def check_imad_output(inputs, output, coefficients, iterations) -> dict:
    """Exact int32 wrap-around chains x <- a*x + b_c (mod 2**32)."""
    coeff = coefficients.detach().cpu().long()
    m, c = _affine_power(int(coeff[0]), coeff[1:, None], iterations, 2**32)
    for start in range(0, inputs.shape[1], CHUNK):
        initial = inputs[:, start:start + CHUNK].cpu().long() % 2**32
        # m < 2**32 and initial < 2**32: split m to keep products below 2**63.
        hi, lo = m >> 16, m & 0xFFFF
        value = ((((hi * initial) % 2**32) << 16) + lo * initial + c) % 2**32
        reference = torch.where(value >= 2**31, value - 2**32, value)
        actual = output[:, start:start + CHUNK].cpu().long()
        if not torch.equal(actual, reference):
            raise RuntimeError("Vector INT32 correctness failed: output differs from exact "
                               "wrap-around multiply-add reference")
    return {"correctness": "all elements passed exact modulo-2**32 INT64 reference",
            "max_abs_error": 0, "max_abs_tolerance": 0, "reference_device": "cpu",
            "validation_recurrence": "INT32 multiply-add with wrap-around state"}


# --------------------------------------------------------------------- read
def check_read(src: torch.Tensor, sink: torch.Tensor, block: int) -> dict:
    """Every block sum against FP64 (bench_bandwidth.py:81-110)."""
    max_error = max_tolerance = 0.0
    factor = 2 * torch.finfo(torch.float32).eps * max(1, math.log2(block))
    step = 1 << 20
    for start in range(0, src.numel(), step):
        chunk = src[start:start + step]
        if chunk.numel() % block:
            matrix = torch.zeros((-(-chunk.numel() // block), block), device=src.device,
                                 dtype=src.dtype)
            matrix.view(-1)[:chunk.numel()].copy_(chunk)
        else:
            matrix = chunk.view(-1, block)
        reference = matrix.sum(dim=1, dtype=torch.float64)
        tolerance = matrix.abs().sum(dim=1, dtype=torch.float64) * factor + 1e-6
        actual = sink[start // block:start // block + reference.numel()].double()
        error = (actual - reference).abs()
        if not torch.all(error <= tolerance).item():
            raise AssertionError("Read reduction validation failed: non-finite or inaccurate "
                                 f"output; max_abs_error={error.max().item():.6g}")
        max_error = max(max_error, error.max().item())
        max_tolerance = max(max_tolerance, tolerance.max().item())
    return {"correctness": "passed (all block sums against FP64, plus masked tail)",
            "max_abs_error": max_error, "max_abs_tolerance": max_tolerance,
            "reference_device": str(src.device)}
