"""ctypes binding of libtcb.so, the sm_100a probe library (include/tcb.h).

The library is the only implementation of the probe kernels: there is no
Python or PyTorch fallback.  If it is missing or cannot be loaded, every call
raises :class:`NativeLibraryError`.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
import os
from pathlib import Path
import threading

LIBRARY_PATH = Path(__file__).resolve().parent / "libtcb.so"

# Status codes (include/tcb.h).
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_RESOURCE = -3
ERR_LAUNCH = -4
ERR_DEVICE = -5
ERR_TIMEOUT = -6
ERR_ALIGNMENT = -7
ERR_SCRATCH_LIMIT = -8

COPY_LDG128, COPY_BULK = 0, 1
READ_FP32, READ_FP16, READ_BF16 = 0, 1, 2

V_BF16, V_FP16, V_FP32, V_FP64, V_INT8_DP4A, V_INT32_IMAD, V_INT8_MULADD = range(7)
# Where the chains read their coefficients (measured on B200): packed bf16x2/f16x2
# FMAs and DP4A run fastest with them in registers (tcb_vector_chains, device
# memory), the other ops with them passed by value as constant-bank operands
# (tcb_vector_chains_imm).
COEFF_IN_REGISTERS = frozenset({V_BF16, V_FP16, V_INT8_DP4A})

T_BF16, T_FP16, T_TF32, T_FP32, T_FP64, T_INT8, T_FP8E4M3, T_MXF4 = range(8)
TV_TCGEN05, TV_DMMA, TV_SIMT, TV_SIMT_REG = 0, 1, 2, 3

FAMILY_COPY, FAMILY_READ, FAMILY_VECTOR, FAMILY_TENSOR, FAMILY_GEMM = 0, 1, 2, 3, 4

# Every symbol include/tcb.h declares.
EXPORTED_SYMBOLS = (
    "tcb_strerror", "tcb_version", "tcb_device_query", "tcb_copy", "tcb_read",
    "tcb_vector_chains", "tcb_vector_chains_imm", "tcb_tensor_peak", "tcb_gemm", "tcb_mx_scales_packed_bytes",
    "tcb_mx_scales_pack", "tcb_kernel_info", "tcb_gemm_mxf4_noalloc",
    "tcb_selftest_bounded_wait",
)


class NativeLibraryError(RuntimeError):
    """libtcb.so is missing or unusable; the probes have no other implementation."""


class TcbError(RuntimeError):
    """A libtcb entry point returned a negative status."""

    def __init__(self, status: int, call: str):
        self.status = status
        self.call = call
        super().__init__(f"{call} failed: {strerror(status)} (status {status})")

    @property
    def is_capability(self) -> bool:
        """True for an explicit capability rejection (not a runtime failure)."""
        return self.status == ERR_UNSUPPORTED

    @property
    def is_resource(self) -> bool:
        return self.status == ERR_RESOURCE


class DeviceProps(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 256),
        ("major", ctypes.c_int), ("minor", ctypes.c_int),
        ("sm_count", ctypes.c_int),
        ("max_smem_per_block", ctypes.c_int),
        ("max_smem_per_sm", ctypes.c_int),
        ("regs_per_sm", ctypes.c_int),
        ("clock_khz", ctypes.c_int),
        ("mem_clock_khz", ctypes.c_int),
        ("mem_bus_width", ctypes.c_int),
        ("l2_cache_bytes", ctypes.c_longlong),
        ("total_mem_bytes", ctypes.c_longlong),
        ("free_mem_bytes", ctypes.c_longlong),
        ("driver_version", ctypes.c_int), ("runtime_version", ctypes.c_int),
    ]


class KernelInfo(ctypes.Structure):
    _fields_ = [
        ("registers_per_thread", ctypes.c_int),
        ("local_bytes_per_thread", ctypes.c_int),
        ("static_smem_bytes", ctypes.c_int),
        ("dynamic_smem_bytes", ctypes.c_int),
        ("max_threads_per_block", ctypes.c_int),
        ("threads_per_block", ctypes.c_int),
        ("tensor_core", ctypes.c_int),
        ("instruction", ctypes.c_char * 128),
        ("execution_kind", ctypes.c_char * 16),
        ("pipeline_stages", ctypes.c_int),
        ("tile_m", ctypes.c_int), ("tile_n", ctypes.c_int),
        ("cluster_ctas", ctypes.c_int),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    override = os.environ.get("TCB_LIBRARY")
    return Path(override) if override else LIBRARY_PATH


def load() -> ctypes.CDLL:
    """Load libtcb.so once (raises NativeLibraryError when unavailable)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise NativeLibraryError(
                f"{path} is missing; build it with `python -m triton_chip_benchmarks_b200.build` "
                "(the probes have no non-CUDA implementation)")
        try:
            lib = ctypes.CDLL(str(path))
        except OSError as exc:
            raise NativeLibraryError(f"cannot load {path}: {exc}") from exc
        vp, i, ll, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t
        lib.tcb_strerror.argtypes, lib.tcb_strerror.restype = [i], ctypes.c_char_p
        lib.tcb_version.argtypes, lib.tcb_version.restype = [], ctypes.c_char_p
        lib.tcb_device_query.argtypes = [i, ctypes.POINTER(DeviceProps)]
        lib.tcb_copy.argtypes = [vp, vp, sz, i, i, i, vp, vp]
        lib.tcb_read.argtypes = [vp, i, ll, vp, i, i, vp]
        lib.tcb_vector_chains.argtypes = [i, vp, vp, vp, ll, i, i, i, i, i, vp]
        lib.tcb_vector_chains_imm.argtypes = [i, vp, vp, vp, ll, i, i, i, i, i, vp]
        lib.tcb_tensor_peak.argtypes = [i, i, vp, vp, vp, vp, vp, i, i, i, i, i, i, i, vp, vp]
        lib.tcb_gemm.argtypes = [i, vp, vp, vp, vp, vp, i, i, i, i, vp, vp]
        lib.tcb_mx_scales_pack.argtypes = [vp, vp, i, i, vp]
        lib.tcb_gemm_mxf4_noalloc.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, vp, vp]
        lib.tcb_mx_scales_packed_bytes.argtypes = [i, i]
        lib.tcb_selftest_bounded_wait.argtypes = [ll, vp, vp]
        lib.tcb_kernel_info.argtypes = [i, i, i, i, i, i, i, i, ctypes.POINTER(KernelInfo)]
        for name in EXPORTED_SYMBOLS:
            if name not in ("tcb_strerror", "tcb_version"):
                getattr(lib, name).restype = i
        lib.tcb_mx_scales_packed_bytes.restype = ctypes.c_longlong
        _lib = lib
        return lib


def strerror(status: int) -> str:
    try:
        return load().tcb_strerror(status).decode()
    except NativeLibraryError:
        return f"status {status}"


def version() -> str:
    return load().tcb_version().decode()


def check(status: int, call: str) -> None:
    if status != OK:
        raise TcbError(status, call)


def _ptr(tensor_or_ptr) -> int | None:
    if tensor_or_ptr is None:
        return None
    if isinstance(tensor_or_ptr, int):
        return tensor_or_ptr
    return tensor_or_ptr.data_ptr()


def _stream(stream) -> int:
    """cudaStream_t handle of a torch stream (the current stream by default)."""
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


@dataclass
class Device:
    name: str
    major: int
    minor: int
    sm_count: int
    max_smem_per_block: int
    max_smem_per_sm: int
    regs_per_sm: int
    clock_khz: int
    mem_clock_khz: int
    mem_bus_width: int
    l2_cache_bytes: int
    total_mem_bytes: int
    free_mem_bytes: int
    driver_version: int
    runtime_version: int


def device_query(device: int) -> Device:
    props = DeviceProps()
    check(load().tcb_device_query(device, ctypes.byref(props)), "tcb_device_query")
    values = {name: getattr(props, name) for name, _ in DeviceProps._fields_}
    values["name"] = props.name.decode(errors="replace")
    return Device(**values)


def copy(src, dst, nbytes: int, variant: int = COPY_LDG128, blocks: int = 0, threads: int = 0,
         stream=None, *, status=None) -> None:
    """dst[:nbytes] = src[:nbytes]; `status` (int32 device word) receives a
    bulk-ring timeout, if any."""
    check(load().tcb_copy(_ptr(src), _ptr(dst), nbytes, variant, blocks, threads, _ptr(status),
                          _stream(stream)), "tcb_copy")


def read(src, dtype: int, elements: int, sink, block_elems: int, threads: int = 0,
         stream=None) -> None:
    check(load().tcb_read(_ptr(src), dtype, elements, _ptr(sink), block_elems, threads,
                          _stream(stream)), "tcb_read")


def vector_chains(dtype: int, inputs, outputs, coefficients, elements: int, iterations: int,
                  blocks: int, threads: int, elems_per_thread: int, unroll: int,
                  stream=None) -> None:
    """Coefficients on the device -> tcb_vector_chains; in host memory (a CPU
    tensor or numpy array) -> tcb_vector_chains_imm (passed to the kernel by value)."""
    on_device = getattr(coefficients, "is_cuda", False)
    if not on_device and hasattr(coefficients, "is_contiguous") and \
            not coefficients.is_contiguous():
        raise ValueError("host coefficients must be contiguous")
    fn = load().tcb_vector_chains if on_device else load().tcb_vector_chains_imm
    name = "tcb_vector_chains" if on_device else "tcb_vector_chains_imm"
    host_ptr = _ptr(coefficients) if on_device or not hasattr(coefficients, "ctypes") \
        else coefficients.ctypes.data
    check(fn(dtype, _ptr(inputs), _ptr(outputs), host_ptr, elements, iterations, blocks, threads,
             elems_per_thread, unroll, _stream(stream)), name)


def vector_coefficients(dtype: int, on_device, on_host):
    """The coefficient tensor to pass to vector_chains for this op: the device
    copy for the ops that run fastest from registers, else the host copy."""
    return on_device if dtype in COEFF_IN_REGISTERS else on_host


def tensor_peak(dtype: int, variant: int, a, b, c, *, blocks: int, blocks_per_sm: int,
                tile_m: int, tile_n: int, tile_k: int, chains: int, iterations: int,
                scale_a=None, scale_b=None, status=None, stream=None) -> None:
    check(load().tcb_tensor_peak(dtype, variant, _ptr(a), _ptr(b), _ptr(scale_a), _ptr(scale_b),
                                 _ptr(c), blocks, blocks_per_sm, tile_m, tile_n, tile_k, chains,
                                 iterations, _ptr(status), _stream(stream)), "tcb_tensor_peak")


def gemm(dtype: int, a, b, c, m: int, n: int, k: int, *, scale_a=None, scale_b=None,
         blocks: int = 0, status=None, stream=None) -> None:
    check(load().tcb_gemm(dtype, _ptr(a), _ptr(b), _ptr(scale_a), _ptr(scale_b), _ptr(c), m, n, k,
                          blocks, _ptr(status), _stream(stream)), "tcb_gemm")


def mx_scales_packed_bytes(rows: int, groups: int) -> int:
    """Bytes of the packed E8M0 layout for scales [rows][groups]."""
    n = load().tcb_mx_scales_packed_bytes(rows, groups)
    check(n if n < 0 else OK, "tcb_mx_scales_packed_bytes")
    return int(n)


def mx_scales_pack(src, dst, rows: int, groups: int, stream=None) -> None:
    check(load().tcb_mx_scales_pack(_ptr(src), _ptr(dst), rows, groups, _stream(stream)),
          "tcb_mx_scales_pack")


def selftest_bounded_wait(limit_ns: int, status, stream=None) -> None:
    """Launch the wait self-test: a bounded wait that cannot succeed, which must
    write ERR_TIMEOUT into `status` and return."""
    check(load().tcb_selftest_bounded_wait(limit_ns, _ptr(status), _stream(stream)),
          "tcb_selftest_bounded_wait")


def kernel_info(family: int, *args: int) -> dict:
    values = list(args) + [0] * (7 - len(args))
    info = KernelInfo()
    check(load().tcb_kernel_info(family, *values[:7], ctypes.byref(info)), "tcb_kernel_info")
    return {
        "registers_per_thread": info.registers_per_thread,
        "local_bytes_per_thread": info.local_bytes_per_thread,
        "static_smem_bytes": info.static_smem_bytes,
        "dynamic_smem_bytes": info.dynamic_smem_bytes,
        "max_threads_per_block": info.max_threads_per_block,
        "threads_per_block": info.threads_per_block,
        "tensor_core": bool(info.tensor_core),
        "instruction": info.instruction.decode(),
        "execution_kind": info.execution_kind.decode(),
        "pipeline_stages": info.pipeline_stages,
        "tile_m": info.tile_m, "tile_n": info.tile_n, "cluster_ctas": info.cluster_ctas,
    }
