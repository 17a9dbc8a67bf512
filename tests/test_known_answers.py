"""The reference's own known-answer tests, restated against this package (CPU).

Each test mirrors one of the reference suite's tests on the same inputs and
verdicts, but drives this package's input builders and checks:
  tests/test_vector_dtypes.py:136-174 (exact low-precision recurrence, FP64
  tolerance scale, naive DP4A recurrence), tests/test_tensor_formats.py:46-53
  (FP4 tiles carry whole MX groups), tests/test_tensor_precision.py:180-187
  (peak tolerance far below one dropped iteration).
"""

from types import SimpleNamespace

import pytest
import torch

from triton_chip_benchmarks_b200 import bench_tensor, bench_vector, validation


def _inputs(dtype, elements, int8_op="dp4a"):
    args = SimpleNamespace(dtype=dtype, inputs="reference", seed=0, int8_op=int8_op)
    return bench_vector.make_inputs(args, elements, torch.device("cpu"))


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_low_precision_recurrence_is_exact_and_identity_is_rejected(dtype):
    inputs, coeff = _inputs(dtype, 31)
    current = inputs.clone()
    for iteration in range(1, 34):
        current = current * coeff[0] + coeff[1:, None]
        info = validation.check_output(inputs, current, coeff, iteration)
        assert info["max_abs_error"] == 0 and info["max_abs_tolerance"] == 0
    with pytest.raises(RuntimeError, match="correctness failed"):
        validation.check_output(inputs, inputs, coeff, 33)


def test_fp64_tolerance_scale_and_corruption():
    inputs, coeff = _inputs("fp64", 31)
    actual = inputs.clone()
    for _ in range(64):
        actual = actual * coeff[0] + coeff[1:, None]
    info = validation.check_output(inputs, actual, coeff, 64)
    assert info["max_abs_tolerance"] < 1e-10
    actual[0, 0] += 1e-8
    with pytest.raises(RuntimeError, match="correctness failed"):
        validation.check_output(inputs, actual, coeff, 64)


def test_int8_check_matches_naive_signed_recurrence():
    inputs, coeff = _inputs("int8", 43)
    weights = validation._signed_bytes(coeff[0].item())
    assert weights == [3, -2, 1, -1]
    actual = inputs.long()
    for iteration in range(1, 4097):
        actual = validation._dot4(actual, weights) + coeff[1:, None].long()
        if iteration in (1, 2, 3, 32, 4096):
            info = validation.check_int8_output(inputs, actual.int(), coeff, iteration)
            assert info["max_abs_error"] == 0
    actual[3, 7] += 1
    with pytest.raises(RuntimeError, match="INT8 correctness failed"):
        validation.check_int8_output(inputs, actual.int(), coeff, 4096)


@pytest.mark.parametrize("inputs", ["reference", "baseline"])
def test_fp4_tiles_carry_whole_mx_groups(inputs):
    configs = bench_tensor.peak_configs("fp4", inputs)
    assert configs
    for config in configs:
        assert config["block_k"] % validation.MX_GROUP_SIZE == 0
        assert config["block_k"] % 2 == 0


@pytest.mark.parametrize("inputs", ["reference", "baseline"])
@pytest.mark.parametrize("key,pass_cols", [("fp32", 1024), ("fp64", 512)])
def test_register_resident_tiles_fit_the_kernel(inputs, key, pass_cols):
    """One k per lane (K <= 32), passes of 32 x (pass_cols / K) outputs, 8 warps."""
    configs = [c for c in bench_tensor.peak_configs(key, inputs) if c["kernel"] == "simt_reg"]
    assert configs
    for config in configs:
        assert config["block_k"] in (8, 16, 32)
        assert config["block_m"] % 32 == 0
        assert config["block_n"] % (pass_cols // config["block_k"]) == 0
        assert config["num_warps"] == 8


def test_reference_mode_sweeps_the_reference_fp32_and_fp64_tiles():
    """bench_tensor.py:497-503 of the reference: FP64 32x32 / 32x64 at K 16, IEEE
    FP32 32x32 / 32x64 / 64x32 / 64x64 at K 32."""
    shapes = {key: {(c["block_m"], c["block_n"], c["block_k"])
                    for c in bench_tensor.peak_configs(key, "reference")}
              for key in ("fp32", "fp64")}
    assert {(32, 32, 16), (32, 64, 16)} <= shapes["fp64"]
    assert {(32, 32, 32), (32, 64, 32), (64, 32, 32), (64, 64, 32)} <= shapes["fp32"]


def test_peak_tolerance_stays_far_below_a_dropped_iteration():
    tolerance = validation.peak_tolerance("bf16", 32, 1024)
    assert tolerance * 64 < 1 / 256
    assert tolerance > 1.9073486328125e-06
    assert validation.peak_tolerance("int8", 64, 1024) == 0.0
