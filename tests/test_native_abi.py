"""The C ABI library loads and exports every symbol include/tcb.h declares (CPU)."""

import ctypes
import re

import pytest

from conftest import REPO

HEADER = REPO / "include" / "tcb.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tcb_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for expected in ("tcb_copy", "tcb_read", "tcb_vector_chains", "tcb_tensor_peak",
                     "tcb_kernel_info", "tcb_device_query", "tcb_strerror", "tcb_version"):
        assert expected in names


def test_library_exports_every_declared_symbol(native):
    lib = ctypes.CDLL(str(native.library_path()))
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing
    assert set(native.EXPORTED_SYMBOLS) >= set(n for n in declared_functions()
                                               if n not in ("tcb_fp4_gemm",))


def test_status_text_and_version(native):
    assert native.version().startswith("tcb ") and "sm_100a" in native.version()
    assert native.strerror(native.OK) == "ok"
    assert "unsupported" in native.strerror(native.ERR_UNSUPPORTED)
    assert "timed out" in native.strerror(native.ERR_TIMEOUT)
    assert native.strerror(-99) == "unknown status"


def test_status_codes_match_header(native):
    text = HEADER.read_text()
    for name in ("OK", "ERR_INVALID_ARGUMENT", "ERR_UNSUPPORTED", "ERR_RESOURCE", "ERR_LAUNCH",
                 "ERR_DEVICE", "ERR_TIMEOUT", "ERR_ALIGNMENT"):
        match = re.search(rf"#define TCB_{name}\s+\(?(-?\d+)\)?", text)
        assert match and int(match.group(1)) == getattr(native, name), name


def test_enums_match_header(native):
    text = HEADER.read_text()
    pairs = {"TCB_T_BF16": native.T_BF16, "TCB_T_MXF4": native.T_MXF4,
             "TCB_T_FP32": native.T_FP32, "TCB_V_INT8_DP4A": native.V_INT8_DP4A,
             "TCB_V_INT8_MULADD": native.V_INT8_MULADD, "TCB_TV_SIMT": native.TV_SIMT,
             "TCB_TV_SIMT_REG": native.TV_SIMT_REG,
             "TCB_COPY_BULK": native.COPY_BULK, "TCB_READ_BF16": native.READ_BF16,
             "TCB_FAMILY_TENSOR": native.FAMILY_TENSOR}
    for name, value in pairs.items():
        match = re.search(rf"#define {name}\s+(\d+)", text)
        assert match and int(match.group(1)) == value, name


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    from triton_chip_benchmarks_b200 import _native
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setenv("TCB_LIBRARY", str(tmp_path / "absent.so"))
    with pytest.raises(_native.NativeLibraryError):
        _native.load()
    monkeypatch.delenv("TCB_LIBRARY")


def test_mx_scales_packed_bytes_matches_oracle(native):
    """Host-side size of the packed scale layout (no GPU call)."""
    import numpy as np
    from oracle import tensor as oracle_tensor
    for rows, groups in ((1, 1), (128, 8), (130, 17), (256, 256), (8192, 256)):
        expected = oracle_tensor.pack_mx_scales(np.zeros((rows, groups), np.uint8)).size
        assert native.mx_scales_packed_bytes(rows, groups) == expected
    with pytest.raises(native.TcbError):
        native.mx_scales_packed_bytes(0, 8)


def test_integration_binding_stub_matches_the_header():
    """The reference-side ctypes stub imports and names only declared entry points."""
    import inspect
    from triton_chip_benchmarks_b200 import tcb_binding
    used = set(re.findall(r"_lib\.(tcb_[a-z_0-9]+)", inspect.getsource(tcb_binding)))
    assert used and used <= set(declared_functions()), used - set(declared_functions())
    for name in ("launch_copy", "launch_read", "launch_vector", "_launch_peak", "_launch"):
        assert callable(getattr(tcb_binding, name))


def test_integration_stub_derives_once_per_tensor_not_per_address(native):
    """The stub's _once cache (host coefficients, K-contiguous B) follows the tensor
    object: reused while the tensor lives unchanged, rebuilt after an in-place change,
    and dropped with the tensor, so a new tensor at a recycled address never sees a
    stale entry.  Runs the stub against the built library (no device needed)."""
    import torch
    from triton_chip_benchmarks_b200 import tcb_binding
    once, derived = tcb_binding._once, tcb_binding._derived
    derived.clear()
    calls = []

    def make(t):
        calls.append(1)
        return t.clone()

    t = torch.arange(8.0)
    first = once(t, make)
    assert once(t, make) is first and len(calls) == 1
    t.add_(1)
    assert torch.equal(once(t, make), t) and len(calls) == 2
    del t, first
    assert not derived
    u = torch.arange(8.0)
    assert torch.equal(once(u, make), u) and len(calls) == 3 and len(derived) == 1


def test_entry_points_reject_bad_arguments_before_touching_a_device(native):
    """Argument validation returns a status without any CUDA call (runs without a GPU)."""
    lib = native.load()
    fake = 0x1000  # never dereferenced: every call below is rejected before a launch
    # Zero bytes is a no-op; null buffers and unknown variants are invalid.
    assert lib.tcb_copy(None, None, 0, native.COPY_BULK, 0, 0, None, None) == native.OK
    assert lib.tcb_copy(None, fake, 64, native.COPY_BULK, 0, 0, None, None) == native.ERR_INVALID_ARGUMENT
    assert lib.tcb_copy(fake, fake, 64, 9, 0, 0, None, None) == native.ERR_INVALID_ARGUMENT
    # Vector chains: elements must equal blocks x threads x elements per thread.
    coeff = (ctypes.c_float * 9)()
    for fn, c in ((lib.tcb_vector_chains, fake), (lib.tcb_vector_chains_imm,
                                                    ctypes.addressof(coeff))):
        assert fn(native.V_FP32, fake, fake, c, 1000, 4, 2, 128, 2, 4, None) == \
            native.ERR_INVALID_ARGUMENT
        assert fn(native.V_FP32, fake, fake, c, 512, 4, 2, 100, 2, 4, None) == \
            native.ERR_INVALID_ARGUMENT
    assert lib.tcb_vector_chains_imm(native.V_FP32, fake, fake, None, 512, 4, 2, 128, 2, 4,
                                     None) == native.ERR_INVALID_ARGUMENT
    # GEMM: a bf16 row of 60 elements is not a whole number of 16-byte TMA units.
    assert lib.tcb_gemm(native.T_BF16, fake, fake, None, None, fake, 128, 128, 60, 0, None,
                        None) == native.ERR_UNSUPPORTED
    assert lib.tcb_gemm(native.T_BF16, None, fake, None, None, fake, 128, 128, 64, 0, None,
                        None) == native.ERR_INVALID_ARGUMENT
    assert lib.tcb_gemm(native.T_MXF4, fake, fake, None, None, fake, 256, 256, 256, 0, None,
                        None) == native.ERR_INVALID_ARGUMENT  # MX FP4 needs its scales
    assert lib.tcb_mx_scales_pack(None, fake, 128, 8, None) == native.ERR_INVALID_ARGUMENT
    # Resident probe: at least one block and one iteration.
    assert lib.tcb_tensor_peak(native.T_FP64, native.TV_DMMA, fake, fake, None, None, fake, 0, 1,
                               128, 128, 16, 1, 1, None, None) == native.ERR_INVALID_ARGUMENT
    assert lib.tcb_kernel_info(99, 0, 0, 0, 0, 0, 0, 0, None) == native.ERR_INVALID_ARGUMENT


def test_vector_coefficient_source_per_op(native):
    """Packed bf16/fp16 and DP4A chains take device coefficients (registers);
    the other ops take the host copy (passed by value, constant bank)."""
    on_device, on_host = object(), object()
    for code in (native.V_BF16, native.V_FP16, native.V_INT8_DP4A):
        assert native.vector_coefficients(code, on_device, on_host) is on_device
    for code in (native.V_FP32, native.V_FP64, native.V_INT32_IMAD, native.V_INT8_MULADD):
        assert native.vector_coefficients(code, on_device, on_host) is on_host
