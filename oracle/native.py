"""ctypes wrapper of the C restatement (tcb_oracle.c) - test infrastructure.

The shared object is built by :func:`build` with gcc into ``oracle/_build``;
it is built on first use when missing.
"""

from __future__ import annotations

import ctypes
from pathlib import Path
import subprocess
import threading

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "tcb_oracle.c"
BUILD_DIR = HERE / "_build"
LIBRARY = BUILD_DIR / "liboracle.so"

_lock = threading.Lock()
_lib = None


def build() -> Path:
    """Compile tcb_oracle.c (strict IEEE: no fast-math, FMA contraction off)."""
    BUILD_DIR.mkdir(exist_ok=True)
    if LIBRARY.exists() and LIBRARY.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIBRARY
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-o", str(LIBRARY), str(SOURCE), "-lm", "-lpthread"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return LIBRARY


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            handle = ctypes.CDLL(str(LIBRARY))
            vp, ll, i, sz = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_size_t
            handle.oracle_copy.argtypes, handle.oracle_copy.restype = [vp, vp, sz, i], i
            for name in ("oracle_chain_f32", "oracle_chain_f64", "oracle_chain_dp4a",
                         "oracle_chain_imad", "oracle_chain_i8"):
                getattr(handle, name).argtypes = [vp, vp, ll, vp, i]
                getattr(handle, name).restype = None
            handle.oracle_chain_h16.argtypes = [vp, vp, ll, vp, i, i]
            handle.oracle_chain_h16.restype = i
            handle.oracle_block_sums.argtypes = [vp, ll, i, vp, vp]
            handle.oracle_block_sums.restype = None
            _lib = handle
        return _lib


def _p(array: np.ndarray) -> int:
    return array.ctypes.data


def copy(src: np.ndarray, dst: np.ndarray, threads: int) -> int:
    """Multi-threaded host copy; returns the threads used."""
    assert src.nbytes == dst.nbytes and src.flags.c_contiguous and dst.flags.c_contiguous
    return lib().oracle_copy(_p(src), _p(dst), src.nbytes, threads)


def chain(kind: str, inputs: np.ndarray, coeff: np.ndarray, iterations: int) -> np.ndarray:
    """Replay 8 chains of [8, elements] inputs step by step (single rounding per step).

    kind: f32, f64, f16, bf16 (16-bit patterns as uint16), dp4a, imad (int32), i8 (int8).
    """
    inputs = np.ascontiguousarray(inputs)
    coeff = np.ascontiguousarray(coeff)
    assert inputs.shape[0] == 8 and coeff.shape == (9,)
    out = np.empty_like(inputs)
    elements = inputs.shape[1]
    handle = lib()
    if kind in ("f16", "bf16"):
        status = handle.oracle_chain_h16(_p(inputs), _p(out), elements, _p(coeff), iterations,
                                         1 if kind == "bf16" else 0)
        if status != 0:
            raise ArithmeticError("x*a+b was not exact in double; replay would double-round")
        return out
    fn = {"f32": handle.oracle_chain_f32, "f64": handle.oracle_chain_f64,
          "dp4a": handle.oracle_chain_dp4a, "imad": handle.oracle_chain_imad,
          "i8": handle.oracle_chain_i8}[kind]
    fn(_p(inputs), _p(out), elements, _p(coeff), iterations)
    return out


def block_sums(src: np.ndarray, block: int) -> tuple[np.ndarray, np.ndarray]:
    src = np.ascontiguousarray(src, dtype=np.float32)
    blocks = -(-src.size // block)
    sums = np.empty(blocks, dtype=np.float64)
    abs_sums = np.empty(blocks, dtype=np.float64)
    lib().oracle_block_sums(_p(src), src.size, block, _p(sums), _p(abs_sums))
    return sums, abs_sums
