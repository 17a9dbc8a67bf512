"""Tensor-probe oracle and product checks pinned to the reference's golden vectors (CPU)."""

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import tensor as oracle_tensor
from triton_chip_benchmarks_b200 import validation
from triton_chip_benchmarks_b200.bench_tensor import precision_descriptor, rates

G = json.loads((GOLDEN / "tensor.json").read_text())
ARR = np.load(GOLDEN / "tensor_inputs.npz")


def test_e2m1_constants():
    assert list(oracle_tensor.E2M1_VALUES) == G["E2M1_VALUES"]
    assert list(validation.E2M1_VALUES) == G["E2M1_VALUES"]
    assert oracle_tensor.MX_GROUP_SIZE == G["MX_GROUP_SIZE"] == validation.MX_GROUP_SIZE
    assert oracle_tensor.E8M0_UNIT_SCALE == G["E8M0_UNIT_SCALE"] == validation.E8M0_UNIT_SCALE
    assert oracle_tensor.FP4_PACKING_FACTOR == G["FP4_PACKING_FACTOR"]


@pytest.mark.parametrize("case", range(3))
def test_e2m1_packing(case):
    entry = G["pack_cases"][case]
    codes = np.array(entry["codes"], dtype=np.uint8)
    assert oracle_tensor.pack_e2m1_pairs(codes).tolist() == entry["packed"]
    assert validation.pack_e2m1_pairs(torch.from_numpy(codes)).tolist() == entry["packed"]
    assert np.array_equal(oracle_tensor.unpack_e2m1(np.array(entry["packed"], dtype=np.uint8)),
                          codes)


def test_e2m1_pack_known_answer():
    # [[1, 2, 9, 10]] -> [[0x21, 0xA9]]: even index in the low nibble.
    assert G["pack_cases"][0]["packed"] == [[0x21, 0xA9]]


def test_tolerance_grid():
    for dtype, k, it, tol in G["tolerance_grid"]:
        assert oracle_tensor.peak_tolerance(dtype, k, it) == tol
        assert validation.peak_tolerance(dtype, k, it) == tol


def test_validate_peak_verdicts():
    for v in G["validate_peak"]:
        ref = np.array(v["reference"])
        cand = np.array([np.nan if x is None else x for x in v["candidate"]])
        assert oracle_tensor.validate_peak(cand, ref, v["dtype"], v["k"], v["iterations"]) \
            == v["accepted"], v["case"]
        tdtype = torch.int32 if v["dtype"] == "int8" else torch.float64 if v["dtype"] == "fp64" \
            else torch.float32
        tc, tr = torch.tensor(cand).to(tdtype), torch.tensor(ref).to(tdtype)
        try:
            validation.validate_peak(tc, tr, v["dtype"], v["k"], v["iterations"])
            accepted = True
        except AssertionError:
            accepted = False
        assert accepted == v["accepted"], v["case"]


def test_rates_and_descriptors():
    for entry in G["rates"]:
        assert rates(entry["ops"], entry["timing"], entry["dtype"]) == entry["result"]
    for key, expected in G["descriptors"].items():
        dtype, precision = key.split(":")
        got = precision_descriptor(dtype, None if precision == "None" else precision)
        if dtype == "fp4":
            # Same fields; the instruction that performs the scaled dot differs by design.
            assert got.pop("dot_operation") != expected.pop("dot_operation")
        assert got == expected


@pytest.mark.parametrize("name", ["bf16", "fp16", "fp32", "int8", "fp64", "fp8"])
def test_resident_reference_matches_reference(name):
    a, b_kn, ref = ARR[f"{name}_a"], ARR[f"{name}_b_kn"], ARR[f"{name}_ref"]
    k = a.shape[-1]
    iterations = 8
    dtype = {"bf16": "bf16", "fp16": "fp16", "fp32": "fp32", "int8": "int8", "fp64": "fp64",
             "fp8": "fp8"}[name]
    for chain in range(2):
        b_nk = np.swapaxes(b_kn[chain], -1, -2)
        got = oracle_tensor.resident_reference(a, b_nk, iterations, dtype)
        assert np.array_equal(got.astype(np.float64), ref[chain].astype(np.float64))
        assert oracle_tensor.validate_peak(got, ref[chain], dtype, k, iterations)
    # The product's validation computes the same exact product.
    prod = validation.reference_product(torch.from_numpy(a) if name != "fp8" else
                                        torch.from_numpy(a).to(torch.float8_e4m3fn),
                                        torch.from_numpy(np.swapaxes(b_kn[0], -1, -2).copy())
                                        .to(torch.from_numpy(a).dtype if name != "fp8"
                                            else torch.float8_e4m3fn))
    assert np.array_equal((prod.double() * iterations).numpy(), ref[0].astype(np.float64))


def test_reference_operand_sets():
    # Ternary / 16 for the float formats, ternary ints, one-hot fp8 rows.
    for name in ("bf16", "fp16", "fp32", "fp64"):
        assert set(np.unique(ARR[f"{name}_a"] * 16)) <= {-1.0, 0.0, 1.0}
    assert set(np.unique(ARR["int8_a"])) <= {-1, 0, 1}
    fp8_a = ARR["fp8_a"]
    assert np.all((fp8_a != 0).sum(-1) == 1) and set(np.unique(fp8_a)) <= {0.0, 1 / 16}
    assert set(np.unique(ARR["fp8_b_kn"] * 16)) <= {-1.0, 1.0}


def test_fp4_inputs_decode_and_reference():
    a, b_kn = ARR["fp4_a_packed"], ARR["fp4_b_packed_kn"]
    va, vb = ARR["fp4_values_a"], ARR["fp4_values_b"]
    assert np.array_equal(oracle_tensor.decode_e2m1(a), va)
    b_nk = np.swapaxes(b_kn, -1, -2)  # [chains, blocks, N, K/2], packed along K
    assert np.array_equal(np.swapaxes(oracle_tensor.decode_e2m1(b_nk), -1, -2), vb)
    assert set(np.unique(va)) <= {-1.0, -0.5, 0.5, 1.0}
    assert np.all(ARR["fp4_scale_a"] == 127) and np.all(ARR["fp4_scale_b"] == 127)
    for chain in range(2):
        got = oracle_tensor.resident_reference(a, b_nk[chain], 1, "fp4", ARR["fp4_scale_a"],
                                               ARR["fp4_scale_b"])
        assert np.array_equal(got, ARR["fp4_ref"][chain])
    torch_vals = validation.decode_e2m1(torch.from_numpy(a))
    assert np.array_equal(torch_vals.numpy(), va)


def test_fp4_scale_semantics():
    assert oracle_tensor.e8m0_value(127) == 1.0
    assert oracle_tensor.e8m0_value(128) == 2.0
    a = ARR["fp4_a_packed"]
    b_nk = np.swapaxes(ARR["fp4_b_packed_kn"], -1, -2)[0]
    base = oracle_tensor.resident_reference(a, b_nk, 1, "fp4", ARR["fp4_scale_a"],
                                            ARR["fp4_scale_b"])
    doubled = oracle_tensor.resident_reference(a, b_nk, 1, "fp4", ARR["fp4_scale_a"] + 1,
                                               ARR["fp4_scale_b"])
    assert np.array_equal(doubled, 2 * base)


def _fp32_answer(a, answer):
    if answer == "tf32":
        return oracle_tensor.tf32_truncate(a)
    if answer == "bf16":
        return torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    return a


def test_fp32_probe_verdicts():
    """The oracle's expected probe answers reproduce the reference's accept/reject."""
    for v in G["fp32_probe_verdicts"]:
        a, expected = oracle_tensor.fp32_probe_expected(v["precision"], 32, 32, 32)
        observed = _fp32_answer(a, v["answer"]) @ np.eye(32, dtype=np.float32)
        assert np.array_equal(observed, expected) == v["accepted"], v


def test_fp64_probe_verdicts():
    a, expected = oracle_tensor.fp64_probe_expected(32, 32, 16)
    answers = {"exact": a, "fp32": a.astype(np.float32).astype(np.float64),
               "permuted": a[::-1]}
    for v in G["fp64_probe_verdicts"]:
        observed = np.zeros((32, 32))
        observed[:, :16] = answers[v["answer"]]
        assert np.array_equal(observed, expected) == v["accepted"], v


def _packed_offset(r: int, g: int, groups_p: int) -> int:
    return (((r // 128) * (groups_p // 8) + g // 8) * 1024 + (g % 8 // 4) * 512 + (r % 32) * 16
            + (r % 128 // 32) * 4 + g % 4)


def test_pack_mx_scales_layout():
    """Packed scale layout: 1 KB per 128 rows x 8 groups, two 32 x 16-byte halves."""
    rows, groups = 256, 16
    src = np.arange(rows * groups, dtype=np.int64).reshape(rows, groups) % 251
    packed = oracle_tensor.pack_mx_scales(src.astype(np.uint8)).reshape(-1)
    for r, g in ((0, 0), (5, 3), (127, 7), (128, 8), (200, 13), (255, 15), (33, 4), (97, 6)):
        assert packed[_packed_offset(r, g, groups)] == src[r, g] % 256
    # Lane l's 16 bytes of a half are rows l, 32+l, 64+l, 96+l, four groups each.
    half = packed[512:1024].reshape(32, 4, 4)
    assert np.array_equal(half[7, 2], src[64 + 7, 4:8] % 256)


def test_pack_mx_scales_padding():
    """Ragged scales pad to 256 rows x 8 groups with the unit scale."""
    src = np.full((130, 17), 3, dtype=np.uint8)
    packed = oracle_tensor.pack_mx_scales(src)
    assert packed.size == 256 * 24
    assert np.count_nonzero(packed == 3) == 130 * 17
    assert np.all(packed[packed != 3] == oracle_tensor.E8M0_UNIT_SCALE)
    # row 129 (lane 1 of quarter 0, row block 1), groups 16 and 17 (block 2, half 0)
    assert packed[_packed_offset(129, 16, 24)] == 3
    assert packed[(1 * 3 + 2) * 1024 + 1 * 16 + 0] == 3
    assert packed[_packed_offset(129, 17, 24)] == 127


def test_gemm_inputs_pad_unaligned_k():
    """Rows that are not whole 16-byte units are zero-padded; aligned K is untouched."""
    from triton_chip_benchmarks_b200.bench_tensor import gemm_inputs, gemm_padded_k
    assert gemm_padded_k("int8", 1000) == 1008 and gemm_padded_k("fp4", 1000) == 1024
    assert gemm_padded_k("bf16", 1000) == 1000 and gemm_padded_k("fp64", 37) == 37
    gen = torch.Generator().manual_seed(0)
    a, b, _ = gemm_inputs("int8", 4, 3, 1000, torch.device("cpu"), gen)
    assert a.shape == (4, 1008) and b.shape == (3, 1008)
    assert not a[:, 1000:].any() and not b[:, 1000:].any()
    a, b, _ = gemm_inputs("bf16", 4, 3, 1000, torch.device("cpu"), gen)
    assert a.shape == (4, 1000)


def test_status_messages_keep_the_reference_classification(native):
    """The library's status messages are the ones the fixture recorded, and the
    reference's _unsupported_reason (bench_tensor.py:94-142) accepts exactly
    TCB_ERR_UNSUPPORTED's as a capability rejection: its sweep records such a tile
    as unsupported and goes on, while every other failure is re-raised."""
    lib = native.load()
    rows = G["status_classification"]
    assert {row["status"] for row in rows} == set(range(-7, 0))
    for row in rows:
        assert lib.tcb_strerror(row["status"]).decode() == row["message"]
        assert (row["reason"] is not None) == (row["status"] == native.ERR_UNSUPPORTED)
