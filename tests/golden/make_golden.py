#!/usr/bin/env python3
"""Generate the golden fixtures in this directory from the reference suite.

Imports the reference suite's own Python modules (bench_tensor, bench_vector,
bench_bandwidth, suite_report, common) read-only from REFERENCE_ROOT
(default: a `reference` checkout beside this repository) and records what they
compute or decide:

  tensor.json / tensor_inputs.npz  E2M1 table and packing, tolerances, validate
                                   verdicts, operand sets and exact references
  vector.npz / vector.json         operand sets, accepted outputs, check verdicts,
                                   operation counts
  bandwidth.json                   read-check verdicts
  suite.json                       summarize() rows and format_table() text
  timing.json                      measure() results on the deterministic fake device

Outputs the reference accepts are produced by this repository's CPU oracle and
then submitted to the reference's checks; a fixture is written only if the
reference accepts the oracle's answer and rejects the planted mistakes.
Run: python tests/golden/make_golden.py
"""

from __future__ import annotations

import io
import json
import os
from pathlib import Path
import sys
from contextlib import redirect_stdout
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REFERENCE_ROOT = Path(os.environ.get("REFERENCE_ROOT", str(REPO.parent / "reference")))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))
sys.path.insert(0, str(REFERENCE_ROOT))

import common as ref_common  # noqa: E402  (reference)
import bench_tensor as ref_tensor  # noqa: E402
import bench_vector as ref_vector  # noqa: E402
import bench_bandwidth as ref_bandwidth  # noqa: E402
import suite_report as ref_report  # noqa: E402

from fake_device import SCENARIOS, FakeDeviceAPI, make_args  # noqa: E402
from oracle import native as oracle_native  # noqa: E402
from oracle import vector as oracle_vector  # noqa: E402


def install_fake_flag_gems(api=None):
    """The reference reaches devices only through flag_gems; give it a CPU stand-in."""
    runtime = SimpleNamespace(device=SimpleNamespace(support_fp64=False, support_bf16=True),
                              torch_device_fn=api, torch_backend_device=None)
    ref_common.flag_gems = SimpleNamespace(device="cuda", vendor_name="nvidia",
                                           runtime=runtime, __version__="fake")


def raises(fn) -> bool:
    try:
        fn()
    except Exception:  # noqa: BLE001
        return True
    return False


# ------------------------------------------------------------------ tensor
def tensor_fixtures():
    install_fake_flag_gems()
    out = {"E2M1_VALUES": list(ref_tensor.E2M1_VALUES),
           "FP4_PACKING_FACTOR": ref_tensor.FP4_PACKING_FACTOR,
           "MX_GROUP_SIZE": ref_tensor.MX_GROUP_SIZE,
           "E8M0_UNIT_SCALE": ref_tensor.E8M0_UNIT_SCALE}
    torch.manual_seed(0)
    pack_cases = [[[1, 2, 9, 10]], torch.randint(0, 16, (4, 16)).tolist(),
                  torch.randint(0, 16, (2, 3, 8)).tolist()]
    out["pack_cases"] = [{"codes": c, "packed": ref_tensor._pack_e2m1_pairs(
        torch.tensor(c, dtype=torch.uint8)).tolist()} for c in pack_cases]
    grid = []
    for dtype in ("bf16", "fp16", "fp32", "int8", "fp64", "fp8", "fp4"):
        for k in (16, 32, 64, 128, 256):
            for it in (1, 64, 1024, 4096, 262144):
                grid.append([dtype, k, it, ref_tensor._peak_tolerance(dtype, k, it)])
    out["tolerance_grid"] = grid
    # validate_peak verdicts on planted candidates.
    verdicts = []
    gen = torch.Generator().manual_seed(1)
    for dtype, k, it in (("bf16", 32, 1024), ("fp64", 16, 1024), ("int8", 64, 1024),
                         ("fp4", 128, 4096), ("fp8", 64, 4096)):
        ref = (torch.randint(-64, 65, (2, 1, 8, 8), generator=gen).double() / 256) * it
        ref = ref.to(torch.int32) if dtype == "int8" else \
            ref if dtype == "fp64" else ref.float()
        tol = ref_tensor._peak_tolerance(dtype, k, it)
        cands = {"exact": ref.clone()}
        if dtype != "int8":
            half = ref.clone()
            half.view(-1)[3] += tol * 0.5
            cands["within_tolerance"] = half
            drop = ref.clone()
            drop.view(-1)[5] -= ref.view(-1)[5] / it + 1.0 / 256
            cands["dropped_iteration"] = drop
            nan = ref.clone()
            nan.view(-1)[0] = float("nan")
            cands["nan"] = nan
        else:
            off = ref.clone()
            off.view(-1)[2] += 1
            cands["off_by_one"] = off
        for name, cand in cands.items():
            ok = not raises(lambda: ref_tensor._validate_peak(cand, ref, dtype, k, it))
            verdicts.append({"dtype": dtype, "k": k, "iterations": it, "case": name,
                             "reference": ref.double().flatten().tolist(),
                             "candidate": [None if v != v else v
                                           for v in cand.double().flatten().tolist()],
                             "accepted": ok})
    out["validate_peak"] = verdicts
    out["rates"] = [
        {"ops": ops, "timing": timing, "dtype": dtype,
         "result": ref_tensor._rates(ops, timing, dtype)}
        for ops, timing, dtype in ((2 * 64 * 64 * 32 * 1024 * 2 * 148, {"median_ms": 1.5,
                                                                       "min_ms": 1.25}, "bf16"),
                                   (10**12, {"median_ms": 2.0, "min_ms": 1.0}, "int8"),
                                   (10**10, {"median_ms": 0.5}, "fp64"))]
    out["descriptors"] = {f"{d}:{p}": ref_tensor._precision_descriptor(d, p)
                          for d, p in (("bf16", None), ("fp16", None), ("fp32", "ieee"),
                                       ("fp32", "tf32"), ("int8", None), ("fp64", None),
                                       ("fp8", None), ("fp4", None))}
    # Operand sets and exact references (small blocks).
    arrays = {}
    for name, dtype, k in (("bf16", torch.bfloat16, 32), ("fp16", torch.float16, 32),
                           ("fp32", torch.float32, 32), ("int8", torch.int8, 64),
                           ("fp64", torch.float64, 16), ("fp8", torch.float8_e4m3fn, 64)):
        torch.manual_seed(0)
        config = {"block_m": 64, "block_n": 64, "block_k": k}
        a, b, _ = ref_tensor._peak_inputs(2, config, dtype, "cpu")
        iterations = 8
        refv = ref_tensor._stack2(ref_tensor._reference(a, b[0]), ref_tensor._reference(a, b[1]))
        refv = refv * iterations
        arrays[f"{name}_a"] = a.double().numpy() if dtype != torch.int8 else a.numpy()
        arrays[f"{name}_b_kn"] = b.double().numpy() if dtype != torch.int8 else b.numpy()
        arrays[f"{name}_ref"] = refv.double().numpy() if dtype != torch.int8 else refv.numpy()
    torch.manual_seed(0)
    config = {"block_m": 64, "block_n": 64, "block_k": 128}
    a, b, _, (sa, sb), (va, vb) = ref_tensor._fp4_peak_inputs(1, config, "cpu")
    arrays["fp4_a_packed"] = a.numpy()
    arrays["fp4_b_packed_kn"] = b.numpy()
    arrays["fp4_scale_a"] = sa.numpy()
    arrays["fp4_scale_b"] = sb.numpy()
    arrays["fp4_values_a"] = va.numpy()
    arrays["fp4_values_b"] = vb.numpy()
    arrays["fp4_ref"] = ref_tensor._stack2(va.matmul(vb[0]), va.matmul(vb[1])).numpy()
    np.savez_compressed(HERE / "tensor_inputs.npz", **arrays)
    # Precision-probe verdicts: the reference probe with its kernel replaced by
    # a function that writes a chosen answer.
    probes = []
    for precision in ("ieee", "tf32"):
        for answer in ("ieee", "tf32", "bf16"):
            def fake_launch(a, b, c, iterations, config, dot_input_precision=None, scales=None,
                            answer=answer):
                x = a[0].float()
                if answer == "tf32":
                    x = torch.from_numpy((x.numpy().view(np.uint32) & np.uint32(0xFFFFE000))
                                         .view(np.float32))
                elif answer == "bf16":
                    x = x.to(torch.bfloat16).float()
                prod = x @ b[0, 0].float()
                c.copy_(torch.stack((prod, prod)).unsqueeze(1))
            ref_tensor._launch_peak, saved = fake_launch, ref_tensor._launch_peak
            try:
                ok = not raises(lambda: ref_tensor._validate_fp32_precision("cpu", precision,
                                                                            "peak"))
            finally:
                ref_tensor._launch_peak = saved
            probes.append({"precision": precision, "answer": answer, "accepted": ok})
    out["fp32_probe_verdicts"] = probes
    fp64 = []
    for answer in ("exact", "fp32", "permuted"):
        def fake_launch(a, b, c, iterations, config, dot_input_precision=None, scales=None,
                        answer=answer):
            x = a[0]
            if answer == "fp32":
                x = x.float().double()
            prod = x @ b[0, 0]
            if answer == "permuted":
                prod = prod.flip(0)
            c.copy_(torch.stack((prod, prod)).unsqueeze(1))
        ref_tensor._launch_peak, saved = fake_launch, ref_tensor._launch_peak
        try:
            ok = not raises(lambda: ref_tensor._validate_fp64_precision("cpu", "peak"))
        finally:
            ref_tensor._launch_peak = saved
        fp64.append({"answer": answer, "accepted": ok})
    out["fp64_probe_verdicts"] = fp64
    out["status_classification"] = status_classification()
    (HERE / "tensor.json").write_text(json.dumps(out, indent=1) + "\n")


def status_classification():
    """The reference's verdict on each libtcb status message raised as RuntimeError.

    _unsupported_reason (bench_tensor.py:94-142) decides whether a failed tile
    is recorded as unsupported (non-null) or re-raised and ends the sweep (null).
    """
    from triton_chip_benchmarks_b200 import _native
    lib = _native.load()
    rows = []
    for status in range(-1, -8, -1):
        message = lib.tcb_strerror(status).decode()
        rows.append({"status": status, "message": message,
                     "reason": ref_tensor._unsupported_reason(RuntimeError(message))})
    return rows


# ------------------------------------------------------------------ vector
def vector_fixtures():
    install_fake_flag_gems()
    arrays, meta = {}, {"cases": [], "throughput": []}
    for dtype, mul_add in (("bf16", False), ("fp16", False), ("fp32", False), ("fp64", False),
                           ("int8", False), ("int8", True)):
        torch.manual_seed(0)
        inputs, coeff = ref_vector._make_inputs(dtype, 256, "cpu", int8_mul_add=mul_add)
        tag = f"{dtype}{'_muladd' if mul_add else ''}"
        arrays[f"{tag}_inputs"] = (inputs.view(torch.int16).numpy() if inputs.dtype in
                                   (torch.bfloat16, torch.float16) else inputs.numpy())
        arrays[f"{tag}_coeff"] = (coeff.view(torch.int16).numpy() if coeff.dtype in
                                  (torch.bfloat16, torch.float16) else coeff.numpy())
        for iterations in (1, 2, 3, 33, 4096):
            if dtype in ("bf16", "fp16"):
                kind = "bf16" if dtype == "bf16" else "f16"
                expected_bits = oracle_native.chain(kind, arrays[f"{tag}_inputs"].view(np.uint16),
                                                    arrays[f"{tag}_coeff"].view(np.uint16),
                                                    iterations)
                expected = torch.from_numpy(expected_bits.view(np.int16)).view(inputs.dtype)
            elif dtype in ("fp32", "fp64"):
                kind = "f32" if dtype == "fp32" else "f64"
                expected = torch.from_numpy(oracle_native.chain(kind, inputs.numpy(),
                                                                coeff.numpy(), iterations))
            elif mul_add:
                expected = torch.from_numpy(oracle_native.chain("i8", inputs.numpy(),
                                                                coeff.numpy(), iterations))
            else:
                expected = torch.from_numpy(oracle_native.chain("dp4a", inputs.numpy(),
                                                                coeff.numpy(), iterations))
            if dtype == "int8" and not mul_add:
                check = lambda out, it=iterations: ref_vector.check_int8_output(  # noqa: E731
                    inputs, out, coeff, it)
            elif mul_add:
                check = lambda out, it=iterations: ref_vector.check_int8_mul_add_output(  # noqa: E731
                    inputs, out, coeff, it)
            else:
                check = lambda out, it=iterations: ref_vector.check_output(  # noqa: E731
                    inputs, out, coeff, it, True)
            if raises(lambda: check(expected)):
                raise SystemExit(f"reference rejected the oracle's {tag} chain at {iterations}")
            planted = expected.clone()
            if planted.dtype.is_floating_point:
                flat = planted.view(-1)
                flat[7] = flat[7] + (0.25 if dtype in ("bf16", "fp16") else 1e-3)
            else:
                planted.view(-1)[7] += 1
            if not raises(lambda: check(planted)):
                raise SystemExit(f"reference accepted a planted {tag} mistake")
            arrays[f"{tag}_out_{iterations}"] = (expected.view(torch.int16).numpy()
                                                 if expected.dtype in (torch.bfloat16,
                                                                       torch.float16)
                                                 else expected.numpy())
            meta["cases"].append({"tag": tag, "iterations": iterations})
    for dtype, elements, iterations, mul_add in (("int8", 17, 32, False), ("fp32", 17, 32, False),
                                                 ("int8", 1024, 4096, True),
                                                 ("bf16", 148 * 1024, 8192, False)):
        timing = {"median_ms": 2.0, "min_ms": 1.0}
        meta["throughput"].append({"dtype": dtype, "elements": elements,
                                   "iterations": iterations, "int8_mul_add": mul_add,
                                   "result": ref_vector.throughput_fields(
                                       dtype, elements, iterations, timing,
                                       int8_mul_add=mul_add)})
    # Tolerance verdicts of the closed-form fp32/fp64 check.
    verdicts = []
    for dtype in ("fp32", "fp64"):
        torch.manual_seed(3)
        inputs, coeff = ref_vector._make_inputs(dtype, 4, "cpu")
        kind = "f32" if dtype == "fp32" else "f64"
        exact = torch.from_numpy(oracle_native.chain(kind, inputs.numpy(), coeff.numpy(), 1000))
        for scale in (0.0, 1e-9, 1e-7, 1e-5, 1e-3):
            cand = exact.clone()
            cand.view(-1)[9] = cand.view(-1)[9] * (1 + scale)
            ok = not raises(lambda: ref_vector.check_output(inputs, cand, coeff, 1000, True))
            verdicts.append({"dtype": dtype, "relative_error": scale, "accepted": ok,
                             "inputs": inputs.double().flatten().tolist(),
                             "coeff": coeff.double().tolist(),
                             "candidate": cand.double().flatten().tolist()})
    meta["closed_form_verdicts"] = verdicts
    np.savez_compressed(HERE / "vector.npz", **arrays)
    (HERE / "vector.json").write_text(json.dumps(meta, indent=1) + "\n")


# --------------------------------------------------------------- bandwidth
def bandwidth_fixtures():
    install_fake_flag_gems()
    out = []
    gen = torch.Generator().manual_seed(2)
    for block in (256, 1024):
        src = torch.randn(block * 2 + 17, generator=gen)
        blocks = -(-src.numel() // block)
        padded = torch.zeros(blocks * block)
        padded[:src.numel()] = src
        exact = padded.view(blocks, block).double().sum(1).float()
        for name, delta in (("exact", 0.0), ("small", 1e-6), ("large", 1.0)):
            sink = exact.clone()
            sink[1] += delta
            ok = not raises(lambda: ref_bandwidth.check_read(src, sink, block))
            out.append({"block": block, "case": name, "src": src.tolist(),
                        "sink": sink.tolist(), "accepted": ok})
    (HERE / "bandwidth.json").write_text(json.dumps(out) + "\n")


# ------------------------------------------------------------------- suite
def suite_documents():
    M = {m.key: m for m in ref_report.METRICS}
    copy_row = lambda mib, peak, eligible=True, smoke=False: {  # noqa: E731
        "pattern": "copy", "peak_gbps": peak, "gbps": peak * 0.99, "buffer_mib": mib,
        "peak_eligible": eligible, "smoke_only": smoke, "cache_regime": "larger_than_l2",
        "block_size": 1024, "num_warps": 4, "timing_method": "graph"}
    read_row = lambda peak: {"pattern": "read", "peak_gbps": peak, "gbps": peak * 0.98,  # noqa: E731
                             "buffer_mib": 2048, "peak_eligible": True}
    tensor_row = lambda peak, **kw: {  # noqa: E731
        "status": "ok", "peak_teraops_per_second": peak, "median_teraops_per_second": peak * 0.99,
        "config": {"block_m": 128, "block_n": 256, "block_k": 64}, "blocks_per_sm": 1,
        "blocks": 148, "iterations": 4096, "measurement_kind": "native_tensor_peak",
        "execution_kind": "tensor", "precision_verified": True,
        "compiled": {"execution_kind": kw.pop("execution_kind", "tensor"),
                     "native_tensor_verified": kw.pop("native", True),
                     "instruction_precision_verified": kw.pop("precision", True),
                     "assembly_audit": "verified"}, **kw}
    vector_row = lambda peak, **kw: {  # noqa: E731
        "status": "ok", "tflops": peak * 0.99, "peak_tflops": peak, "block_size": 512,
        "num_warps": 8, "unroll": 4, "blocks_per_sm": 16, "iterations": 4096,
        "native_arithmetic_verified": kw.pop("native", True), "operation": "FMA", **kw}
    cases = [
        ("memory_capacity", {"status": "ok", "device": {"total_memory_bytes": 191_986_024_448}}),
        ("memory_capacity", {"status": "ok", "device": {}}),
        ("memory_bandwidth", {"status": "ok", "results": [
            copy_row(256, 5000.0, eligible=False), copy_row(2048, 6400.0),
            copy_row(1024, 6300.0), read_row(6900.0)]}),
        ("memory_bandwidth", {"status": "ok", "results": [copy_row(8, 900.0, False, True),
                                                          read_row(1000.0)]}),
        ("memory_bandwidth", {"status": "error", "reason": "boom"}),
        ("tensor_bf16", {"status": "ok", "results": [tensor_row(1500.0), tensor_row(1600.0),
                                                     {"status": "skipped", "reason": "spills"}]}),
        ("tensor_fp32", {"status": "ok", "results": [tensor_row(60.0, execution_kind="simt",
                                                                native=False)]}),
        ("tensor_tf32", {"status": "ok", "results": [tensor_row(700.0, precision=False)]}),
        ("tensor_int8", {"status": "ok", "results": [
            {"status": "ok", "tops": 3000.0, "peak_tops": 3100.0,
             "compiled": {"execution_kind": "tensor", "native_tensor_verified": True,
                          "instruction_precision_verified": True}}]}),
        ("tensor_fp8", {"status": "unsupported", "reason": "no fp8"}),
        ("tensor_fp4", {"status": "ok", "results": [{"status": "unsupported", "reason": "a"},
                                                    {"status": "unsupported", "reason": "b"}]}),
        ("tensor_fp64", {"status": "ok", "results": [{"status": "skipped", "reason": "x"},
                                                     {"status": "unsupported", "reason": "y"}]}),
        ("tensor_fp16", {"status": "ok", "arguments": {"quick": True},
                         "results": [tensor_row(100.0)]}),
        ("tensor_bf16", {"status": "ok", "results": "not-a-list"}),
        ("vector_fp32", {"status": "ok", "results": [vector_row(70.0), vector_row(72.0)]}),
        ("vector_bf16", {"status": "ok", "results": [vector_row(140.0, native=False)]}),
        ("vector_int8", {"status": "ok", "results": [
            {"status": "ok", "tops": 200.0, "peak_tops": 210.0, "native_arithmetic_verified": False,
             "includes_unpacking": True}]}),
        ("vector_fp8", {"status": "not_implemented", "reason": "no native fp8 vector path"}),
        ("vector_fp4", {"status": "unsupported", "reason": "fp4 is not an arithmetic type"}),
        ("vector_fp64", {"status": "ok", "results": [{"status": "ok", "tflops": 0.0,
                                                      "peak_tflops": 1.0}]}),
        ("vector_fp16", {"status": "unavailable", "reason": "no device"}),
    ]
    out = []
    for key, doc in cases:
        out.append({"metric": key, "document": doc,
                    "result": ref_report.summarize(M[key], doc)})
    table_rows = [case["result"] for case in out]
    return {"metrics": [[m.key, m.group, m.precision, m.unit] for m in ref_report.METRICS],
            "cases": out, "table_input": table_rows,
            "table": ref_report.format_table(table_rows),
            "empty": [ref_report.empty_metric(m) for m in ref_report.METRICS]}


# ------------------------------------------------------------------ timing
def timing_fixtures():
    out = {}
    for name, spec in SCENARIOS.items():
        api = FakeDeviceAPI(**spec["api"])
        install_fake_flag_gems(api)
        args = make_args(**spec["args"])
        try:
            with redirect_stdout(io.StringIO()):
                result = ref_common.measure(api.launch, args)
        except RuntimeError as exc:
            out[name] = {"error": type(exc).__name__, "message": str(exc),
                         "launches": api.launches, "replays": api.replays}
            continue
        out[name] = {"result": result, "launches": api.launches, "replays": api.replays,
                     "final_clock_ms": api.now_ms}
    (HERE / "timing.json").write_text(json.dumps(out, indent=1) + "\n")


def main():
    tensor_fixtures()
    vector_fixtures()
    bandwidth_fixtures()
    (HERE / "suite.json").write_text(json.dumps(suite_documents(), indent=1) + "\n")
    timing_fixtures()
    for path in sorted(HERE.glob("*.json")) + sorted(HERE.glob("*.npz")):
        print(f"{path.name}: {path.stat().st_size} bytes")


if __name__ == "__main__":
    main()
