"""tcb_gemm_mxf4_noalloc, the MX FP4 GEMM that allocates nothing (GPU).

Some callers of this library cannot allocate device memory themselves: a
plugin whose host framework hands out all device memory from its own pool, or
a latency-critical path where cudaMalloc/cudaFree (and the synchronisation
they bring) are not allowed.  For them the library offers one MX FP4 GEMM
that takes plain [rows][K/32] E8M0 scales and packs them into a fixed scratch
array of its own instead of into caller-allocated buffers.

This test calls that entry point through the C ABI (ctypes on libtcb.so) and
compares its output with the regular tcb_gemm on scales the test packed into
buffers of its own.  MX FP4 products of E2M1 codes with power-of-two scales
are exact in fp32 here, so the two must agree bit for bit (the tolerance every
FP4 GEMM test uses).  Two calls run back to back with different shapes and
scales, the second smaller than the first, so stale scratch contents from the
first call would show up in the second.  The file is named to be collected
last, so a run stopping at the first failure has run every other test first.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import tensor as oracle_tensor

pytestmark = pytest.mark.gpu

MXF4 = 7


def _lib(native):
    lib = native.load()
    fn = lib.tcb_gemm_mxf4_noalloc
    vp, i = ctypes.c_void_p, ctypes.c_int
    fn.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, vp, vp]
    fn.restype = i
    return lib


def _problem(m, n, k, seed):
    gen = torch.Generator().manual_seed(seed)
    a = torch.from_numpy(oracle_tensor.pack_e2m1_pairs(
        torch.randint(0, 16, (m, k), generator=gen, dtype=torch.uint8).numpy()))
    b = torch.from_numpy(oracle_tensor.pack_e2m1_pairs(
        torch.randint(0, 16, (n, k), generator=gen, dtype=torch.uint8).numpy()))
    sa = torch.randint(124, 131, (m, k // 32), generator=gen, dtype=torch.uint8)
    sb = torch.randint(124, 131, (n, k // 32), generator=gen, dtype=torch.uint8)
    return a, b, sa, sb


def _with_packed_buffers(native, cuda, a, b, sa, sb, m, n, k):
    """The existing path: caller-allocated packed scales + tcb_gemm."""
    groups = k // 32
    psa = torch.empty(native.mx_scales_packed_bytes(m, groups), dtype=torch.uint8, device=cuda)
    psb = torch.empty(native.mx_scales_packed_bytes(n, groups), dtype=torch.uint8, device=cuda)
    native.mx_scales_pack(sa, psa, m, groups)
    native.mx_scales_pack(sb, psb, n, groups)
    c = torch.full((m, n), -7.0, device=cuda)
    native.gemm(MXF4, a, b, c, m, n, k, scale_a=psa, scale_b=psb)
    torch.cuda.synchronize()
    return c.cpu()


def _no_alloc(lib, cuda, a, b, sa, sb, m, n, k):
    c = torch.full((m, n), -7.0, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.tcb_gemm_mxf4_noalloc(a.data_ptr(), b.data_ptr(), sa.data_ptr(), sb.data_ptr(),
                                   c.data_ptr(), m, n, k, 0, status.data_ptr(), stream)
    assert rc == 0, lib.tcb_strerror(rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return c.cpu()


def test_no_alloc_gemm_matches_the_allocating_path_on_two_calls(cuda, native):
    lib = _lib(native)
    # First a CTA-pair problem with ragged edges, then a smaller single-CTA one
    # (M <= 128) whose packed scales cover only part of what the first wrote.
    for m, n, k, seed in ((520, 776, 2048, 1), (96, 264, 544, 2)):
        a, b, sa, sb = (t.to(cuda) for t in _problem(m, n, k, seed))
        expected = _with_packed_buffers(native, cuda, a, b, sa, sb, m, n, k)
        got = _no_alloc(lib, cuda, a, b, sa, sb, m, n, k)
        assert torch.equal(got, expected), f"{m}x{n}x{k}: max err " \
            f"{(got.double() - expected.double()).abs().max().item()}"
        # Both agree with the exact host product as well.
        ref = oracle_tensor.resident_reference(a.cpu().numpy(), b.cpu().numpy(), 1, "fp4",
                                               sa.cpu().numpy(), sb.cpu().numpy())
        assert np.array_equal(got.double().numpy(), ref)


def test_no_alloc_gemm_rejects_problems_beyond_its_scratch(cuda, native):
    lib = _lib(native)
    fake = 0x1000  # never dereferenced: the size check comes before any launch
    # M = N = 32768 at K = 8192: 8 MiB of packed scales per operand, 16 MiB in all.
    rc = lib.tcb_gemm_mxf4_noalloc(fake, fake, fake, fake, fake, 32768, 32768, 8192, 0, None,
                                   None)
    assert rc == native.ERR_SCRATCH_LIMIT
    assert "scratch" in native.strerror(rc)
