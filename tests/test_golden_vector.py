"""Vector-chain oracle and product checks pinned to the reference's golden vectors (CPU)."""

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import native as oracle_native
from oracle import vector as oracle_vector
from triton_chip_benchmarks_b200 import validation

META = json.loads((GOLDEN / "vector.json").read_text())
ARR = np.load(GOLDEN / "vector.npz")
CASES = [(c["tag"], c["iterations"]) for c in META["cases"]]


def _torch(array, tag):
    if tag in ("bf16", "fp16"):
        return torch.from_numpy(array.copy()).view(torch.bfloat16 if tag == "bf16"
                                                   else torch.float16)
    return torch.from_numpy(array.copy())


@pytest.mark.parametrize("tag,iterations", CASES)
def test_oracle_replay_matches_golden(tag, iterations):
    inputs, coeff = ARR[f"{tag}_inputs"], ARR[f"{tag}_coeff"]
    expected = ARR[f"{tag}_out_{iterations}"]
    kind = {"bf16": "bf16", "fp16": "f16", "fp32": "f32", "fp64": "f64", "int8": "dp4a",
            "int8_muladd": "i8"}[tag]
    if kind in ("bf16", "f16"):
        got = oracle_native.chain(kind, inputs.view(np.uint16), coeff.view(np.uint16), iterations)
        assert np.array_equal(got.view(np.int16), expected)
    else:
        assert np.array_equal(oracle_native.chain(kind, inputs, coeff, iterations), expected)


@pytest.mark.parametrize("tag,iterations", CASES)
def test_closed_forms_match_golden(tag, iterations):
    inputs, coeff = ARR[f"{tag}_inputs"], ARR[f"{tag}_coeff"]
    expected = ARR[f"{tag}_out_{iterations}"]
    if tag == "int8":
        assert np.array_equal(oracle_vector.dp4a_reference(inputs, coeff, iterations),
                              expected.astype(np.int64))
    elif tag == "int8_muladd":
        assert np.array_equal(oracle_vector.mod256_reference(inputs, coeff, iterations),
                              expected.astype(np.int64))
    elif tag in ("bf16", "fp16"):
        x = _torch(inputs, tag).double().numpy()
        c = _torch(coeff, tag).double().numpy()
        ref, tol = oracle_vector.closed_form_reference(x, c, iterations)
        assert np.array_equal(_torch(expected, tag).double().numpy(), ref)
    else:
        assert oracle_vector.closed_form_check(inputs, expected, coeff, iterations, tag)


@pytest.mark.parametrize("tag,iterations", CASES)
def test_product_checks_accept_golden_and_reject_mistakes(tag, iterations):
    inputs = _torch(ARR[f"{tag}_inputs"], tag)
    coeff = _torch(ARR[f"{tag}_coeff"], tag)
    expected = _torch(ARR[f"{tag}_out_{iterations}"], tag)
    check = {"int8": validation.check_int8_output,
             "int8_muladd": validation.check_int8_mul_add_output}.get(tag)
    if check is None:
        def check(i, o, c, n):
            return validation.check_output(i, o, c, n, True)
    check(inputs, expected, coeff, iterations)
    planted = expected.clone()
    if planted.dtype.is_floating_point:
        planted.view(-1)[7] += 0.25 if tag in ("bf16", "fp16") else 1e-3
    else:
        planted.view(-1)[7] += 1
    with pytest.raises(RuntimeError):
        check(inputs, planted, coeff, iterations)


def test_product_exact_replay_matches_oracle():
    """check_chain_exact (FP64 replay with one rounding) equals the C oracle for 16/32-bit."""
    rng = np.random.default_rng(0)
    for dtype, kind in ((torch.float32, "f32"), (torch.float16, "f16"), (torch.bfloat16, "bf16")):
        x = torch.from_numpy(rng.uniform(0.5, 1.0, (8, 64))).to(dtype)
        coeff = torch.tensor([0.9990234375] + [0.0009765625] * 8, dtype=dtype)
        if dtype == torch.float32:
            out = oracle_native.chain(kind, x.numpy(), coeff.numpy(), 500)
            out_t = torch.from_numpy(out)
        else:
            bits = oracle_native.chain(kind, x.view(torch.int16).numpy().view(np.uint16),
                                       coeff.view(torch.int16).numpy().view(np.uint16), 500)
            out_t = torch.from_numpy(bits.view(np.int16)).view(dtype)
        result = validation.check_chain_exact(x, out_t, coeff, 500)
        assert result["bit_exact"]


def test_throughput_counting():
    from triton_chip_benchmarks_b200 import bench_vector
    for entry in META["throughput"]:
        per_update = 8 if entry["dtype"] == "int8" and not entry["int8_mul_add"] else 2
        ops = per_update * 8 * entry["elements"] * entry["iterations"]
        key = "counted_integer_ops" if entry["dtype"] == "int8" else "counted_flops"
        assert entry["result"][key] == ops
        assert entry["result"]["ops_per_accumulator_update"] == (per_update if entry["dtype"] ==
                                                                 "int8" else 2)
        assert oracle_vector.counted_operations(entry["dtype"], entry["elements"],
                                                entry["iterations"], entry["int8_mul_add"]) == ops
        args = type("A", (), {"dtype": entry["dtype"],
                              "int8_op": "muladd" if entry["int8_mul_add"] else "dp4a"})()
        assert bench_vector.ops_per_update(args) == per_update


def test_closed_form_tolerance_verdicts():
    for v in META["closed_form_verdicts"]:
        x = np.array(v["inputs"]).reshape(8, -1)
        cand = np.array(v["candidate"]).reshape(8, -1)
        coeff = np.array(v["coeff"])
        assert oracle_vector.closed_form_check(x, cand, coeff, 1000, v["dtype"]) == v["accepted"]
        dtype = torch.float32 if v["dtype"] == "fp32" else torch.float64
        try:
            validation.check_output(torch.from_numpy(x).to(dtype),
                                    torch.from_numpy(cand).to(dtype),
                                    torch.from_numpy(coeff).to(dtype), 1000, True)
            accepted = True
        except RuntimeError:
            accepted = False
        assert accepted == v["accepted"], v["relative_error"]


def test_dp4a_weights_constant():
    # Packed bytes (3, -2, 1, -1) -> 0xFF01FE03 as a signed int32.
    assert oracle_vector.packed_dp4a_weights() == int(ARR["int8_coeff"][0])
    assert oracle_vector._signed_bytes(oracle_vector.packed_dp4a_weights()) == [3, -2, 1, -1]
