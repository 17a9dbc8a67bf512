"""Resident tensor-probe kernels through the C ABI against the exact oracle (GPU).

Operands are small integers scaled by powers of two, so every product and
partial sum is exactly representable: the kernels must match the oracle's
iterations * (A . B^T) bit for bit.
"""

import numpy as np
import pytest
import torch

from oracle import tensor as oracle_tensor

pytestmark = pytest.mark.gpu

BF16, FP16, TF32, FP32, FP64, INT8, FP8, MXF4 = range(8)
TCGEN05, DMMA, SIMT, SIMT_REG = 0, 1, 2, 3
STORAGE = {BF16: torch.bfloat16, FP16: torch.float16, TF32: torch.float32,
           FP32: torch.float32, FP64: torch.float64, INT8: torch.int8,
           FP8: torch.float8_e4m3fn}
NAME = {BF16: "bf16", FP16: "fp16", TF32: "tf32", FP32: "fp32", FP64: "fp64", INT8: "int8",
        FP8: "fp8", MXF4: "fp4"}


def _operands(dtype, blocks, chains, m, n, k, seed):
    gen = torch.Generator().manual_seed(seed)
    if dtype == MXF4:
        a_codes = torch.randint(0, 16, (blocks, m, k), generator=gen, dtype=torch.uint8)
        b_codes = torch.randint(0, 16, (chains, blocks, n, k), generator=gen, dtype=torch.uint8)
        return (torch.from_numpy(oracle_tensor.pack_e2m1_pairs(a_codes.numpy())),
                torch.from_numpy(oracle_tensor.pack_e2m1_pairs(b_codes.numpy())))
    ia = torch.randint(-3, 4, (blocks, m, k), generator=gen)
    ib = torch.randint(-3, 4, (chains, blocks, n, k), generator=gen)
    if dtype == INT8:
        return ia.to(torch.int8), ib.to(torch.int8)
    return (ia.double() / 4).to(STORAGE[dtype]), (ib.double() / 4).to(STORAGE[dtype])


def _host(t):
    if t.dtype == torch.float8_e4m3fn:
        return t.double().numpy()
    if t.dtype == torch.bfloat16:
        return t.double().numpy()
    return t.numpy()


def _run(native, cuda, dtype, variant, a, b, m, n, k, chains, blocks, iterations, bps=1,
         sa=None, sb=None):
    out_dtype = torch.int32 if dtype == INT8 else torch.float64 if dtype == FP64 else torch.float32
    c = torch.full((chains, blocks, m, n), -7, dtype=out_dtype, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    native.tensor_peak(dtype, variant, a.to(cuda), b.to(cuda), c, blocks=blocks,
                       blocks_per_sm=bps, tile_m=m, tile_n=n, tile_k=k, chains=chains,
                       iterations=iterations, scale_a=None if sa is None else sa.to(cuda),
                       scale_b=None if sb is None else sb.to(cuda), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return c.cpu()


def _check(dtype, got, a, b, iterations, sa=None, sb=None):
    chains, blocks = got.shape[0], got.shape[1]
    av = _host(a)
    bv = _host(b)
    for c in range(chains):
        if dtype == MXF4:
            ref = oracle_tensor.resident_reference(
                av, bv[c], iterations, "fp4",
                None if sa is None else sa.numpy(), None if sb is None else sb.numpy())
        else:
            ref = oracle_tensor.resident_reference(av, bv[c], iterations, NAME[dtype])
        assert np.array_equal(got[c].double().numpy(), ref.astype(np.float64)), \
            f"chain {c}: max err {np.abs(got[c].double().numpy() - ref).max()}"


TC_CASES = [
    # dtype, m, n, k, chains
    (BF16, 128, 128, 64, 1), (BF16, 128, 256, 32, 2), (BF16, 256, 256, 64, 1),
    (FP16, 128, 256, 64, 1), (FP16, 256, 256, 128, 1),
    (TF32, 128, 128, 32, 2), (TF32, 256, 256, 32, 1),
    (INT8, 128, 256, 64, 2), (INT8, 256, 256, 128, 1),
    (FP8, 128, 128, 64, 2), (FP8, 256, 256, 128, 1),
    (MXF4, 128, 128, 128, 2), (MXF4, 256, 256, 256, 1), (MXF4, 128, 256, 512, 1),
    # 64-row tiles (one M=64 accumulator, 16 rows per tensor-memory sub-partition),
    # the reference's NVIDIA tile set (bench_tensor.py:504-511) among them.
    (BF16, 64, 64, 32, 2), (BF16, 64, 128, 32, 2), (FP16, 64, 256, 64, 1),
    (TF32, 64, 64, 32, 2), (INT8, 64, 128, 64, 2), (FP8, 64, 64, 64, 2),
]


@pytest.mark.parametrize("dtype,m,n,k,chains", TC_CASES)
@pytest.mark.parametrize("iterations", [1, 3, 64])
def test_tcgen05_exact(cuda, native, dtype, m, n, k, chains, iterations):
    blocks = 3
    a, b = _operands(dtype, blocks, chains, m, n, k, seed=m + n + k + iterations)
    sa = sb = None
    if dtype == MXF4:
        sa = torch.full((blocks, m, k // 32), 127, dtype=torch.uint8)
        sb = torch.full((blocks, n, k // 32), 127, dtype=torch.uint8)
    got = _run(native, cuda, dtype, TCGEN05, a, b, m, n, k, chains, blocks, iterations,
               sa=sa, sb=sb)
    _check(dtype, got, a, b, iterations, sa, sb)


@pytest.mark.parametrize("bps", [2, 4])
def test_tcgen05_blocks_per_sm(cuda, native, bps):
    m, n, k, chains, blocks, iterations = 128, 128, 64, 1, 300, 16
    a, b = _operands(BF16, blocks, chains, m, n, k, seed=bps)
    got = _run(native, cuda, BF16, TCGEN05, a, b, m, n, k, chains, blocks, iterations, bps)
    _check(BF16, got, a, b, iterations)


def test_mxf4_scale_doubling(cuda, native):
    m, n, k, blocks = 128, 128, 128, 2
    a, b = _operands(MXF4, blocks, 1, m, n, k, seed=11)
    sa = torch.full((blocks, m, k // 32), 127, dtype=torch.uint8)
    sb = torch.full((blocks, n, k // 32), 127, dtype=torch.uint8)
    base = _run(native, cuda, MXF4, TCGEN05, a, b, m, n, k, 1, blocks, 1, sa=sa, sb=sb)
    doubled = _run(native, cuda, MXF4, TCGEN05, a, b, m, n, k, 1, blocks, 1, sa=sa + 1, sb=sb)
    assert torch.equal(doubled, 2 * base)


def test_mxf4_per_group_scales(cuda, native):
    """Scale factors that vary by row and by 32-element K group."""
    m, n, k, blocks = 128, 256, 256, 2
    a, b = _operands(MXF4, blocks, 1, m, n, k, seed=5)
    gen = torch.Generator().manual_seed(9)
    sa = torch.randint(125, 130, (blocks, m, k // 32), generator=gen, dtype=torch.uint8)
    sb = torch.randint(125, 130, (blocks, n, k // 32), generator=gen, dtype=torch.uint8)
    got = _run(native, cuda, MXF4, TCGEN05, a, b, m, n, k, 1, blocks, 1, sa=sa, sb=sb)
    _check(MXF4, got, a, b, 1, sa, sb)


@pytest.mark.parametrize("variant,m,n,k,chains", [
    (DMMA, 128, 128, 16, 2), (DMMA, 256, 256, 32, 1), (DMMA, 128, 256, 8, 1),
    (SIMT, 128, 128, 16, 2), (SIMT, 256, 256, 32, 1)])
@pytest.mark.parametrize("iterations", [1, 5])
def test_fp64_exact(cuda, native, variant, m, n, k, chains, iterations):
    blocks = 2
    a, b = _operands(FP64, blocks, chains, m, n, k, seed=k + iterations)
    got = _run(native, cuda, FP64, variant, a, b, m, n, k, chains, blocks, iterations)
    _check(FP64, got, a, b, iterations)


@pytest.mark.parametrize("m,n,k,chains", [(128, 128, 32, 2), (256, 256, 32, 1),
                                          (128, 256, 8, 1)])
@pytest.mark.parametrize("iterations", [1, 7])
def test_fp32_simt_exact(cuda, native, m, n, k, chains, iterations):
    blocks = 2
    a, b = _operands(FP32, blocks, chains, m, n, k, seed=m + iterations)
    got = _run(native, cuda, FP32, SIMT, a, b, m, n, k, chains, blocks, iterations)
    _check(FP32, got, a, b, iterations)


# Register-resident FP32: one k per lane, passes of 32 x (1024 / K) outputs, the
# K partial sums added by a shuffle reduce-scatter; each supported K, pass counts
# above one in both directions, odd pass counts.
@pytest.mark.parametrize("m,n,k,chains", [(64, 64, 32, 2), (128, 128, 32, 2), (256, 256, 32, 1),
                                          (96, 160, 32, 1), (64, 192, 16, 1), (96, 256, 8, 2)])
@pytest.mark.parametrize("iterations", [1, 7])
def test_fp32_simt_reg_exact(cuda, native, m, n, k, chains, iterations):
    blocks = 3
    a, b = _operands(FP32, blocks, chains, m, n, k, seed=n + k + iterations)
    got = _run(native, cuda, FP32, SIMT_REG, a, b, m, n, k, chains, blocks, iterations)
    _check(FP32, got, a, b, iterations)


# FP64 on the same kernel: 8 x 8 lane tiles, passes of 32 x (512 / K); the
# reference's FP64 tiles (32 x 32 and 32 x 64 at K = 16) among them.
@pytest.mark.parametrize("m,n,k,chains", [(32, 32, 16, 2), (32, 64, 16, 2), (64, 64, 32, 1),
                                          (256, 256, 32, 2), (96, 128, 8, 1)])
@pytest.mark.parametrize("iterations", [1, 6])
def test_fp64_simt_reg_exact(cuda, native, m, n, k, chains, iterations):
    blocks = 3
    a, b = _operands(FP64, blocks, chains, m, n, k, seed=m + n + k + iterations)
    got = _run(native, cuda, FP64, SIMT_REG, a, b, m, n, k, chains, blocks, iterations)
    _check(FP64, got, a, b, iterations)


def test_fp32_simt_reg_rejects_unsupported_shapes(cuda, native):
    a = torch.zeros((1, 64, 64), dtype=torch.float32, device=cuda)
    c = torch.zeros((1, 1, 64, 64), device=cuda)
    for (m, n, k, dtype) in [(64, 64, 64, FP32), (48, 64, 32, FP32), (64, 96, 16, FP32),
                             (32, 48, 16, FP64), (64, 64, 32, BF16)]:
        with pytest.raises(native.TcbError) as info:
            native.tensor_peak(dtype, SIMT_REG, a, a, c, blocks=1, blocks_per_sm=1, tile_m=m,
                               tile_n=n, tile_k=k, chains=1, iterations=1)
        assert info.value.is_capability


def test_fp32_precision_probes(cuda):
    from triton_chip_benchmarks_b200 import bench_tensor
    ieee = bench_tensor.validate_fp32_precision(cuda, "ieee")
    tf32 = bench_tensor.validate_fp32_precision(cuda, "tf32")
    assert ieee["passed"] and tf32["passed"]


@pytest.mark.parametrize("variant", [DMMA, SIMT])
def test_fp64_precision_probe(cuda, variant):
    from triton_chip_benchmarks_b200 import bench_tensor
    assert bench_tensor.validate_fp64_precision(cuda, variant)["passed"]


def test_fp4_arithmetic_probe(cuda):
    from triton_chip_benchmarks_b200 import bench_tensor
    assert bench_tensor.validate_fp4_arithmetic(cuda)["scale_sensitivity_verified"]


def test_unsupported_tiles_are_capability_errors(cuda, native):
    """32-row tiles, and 64-row MX FP4 tiles (its scale layout follows M = 128)."""
    a = torch.zeros((1, 64, 256), dtype=torch.uint8, device=cuda)
    c = torch.zeros((1, 1, 64, 64), device=cuda)
    for dtype, m, k in ((BF16, 32, 64), (MXF4, 64, 256)):
        with pytest.raises(native.TcbError) as info:
            native.tensor_peak(dtype, TCGEN05, a, a, c, blocks=1, blocks_per_sm=1, tile_m=m,
                               tile_n=64, tile_k=k, chains=1, iterations=1, scale_a=a,
                               scale_b=a)
        assert info.value.is_capability


def test_kernel_info_reports_instruction(native, cuda):
    info = native.kernel_info(native.FAMILY_TENSOR, BF16, TCGEN05, 256, 256, 64, 1, 1)
    assert "kind::f16" in info["instruction"] and info["execution_kind"] == "tensor"
    assert info["local_bytes_per_thread"] == 0
    simt = native.kernel_info(native.FAMILY_TENSOR, FP32, SIMT, 256, 256, 32, 1, 1)
    assert simt["instruction"] == "fma.rn.f32" and simt["execution_kind"] == "simt"
    reg = native.kernel_info(native.FAMILY_TENSOR, FP32, SIMT_REG, 256, 256, 32, 1, 1)
    assert reg["instruction"] == "fma.rn.f32" and reg["execution_kind"] == "simt"
    assert reg["local_bytes_per_thread"] == 0 and reg["threads_per_block"] == 256
    reg64 = native.kernel_info(native.FAMILY_TENSOR, FP64, SIMT_REG, 32, 64, 16, 2, 1)
    assert reg64["instruction"] == "fma.rn.f64" and reg64["execution_kind"] == "simt"
    assert reg64["local_bytes_per_thread"] == 0


GEMM_CASES = [(BF16, 256, 256, 64), (BF16, 512, 512, 1024), (FP16, 384, 512, 192),
              (TF32, 256, 256, 96), (INT8, 256, 512, 256), (FP8, 256, 256, 512),
              (MXF4, 256, 256, 256), (MXF4, 512, 768, 2048), (MXF4, 128, 256, 8192)]
# Masked tails: M, N not tile multiples, ragged last K block, N % 4 != 0 (element
# stores), single row, and a reference-style odd square size.
GEMM_TAIL_CASES = [(BF16, 200, 300, 320), (BF16, 128, 258, 64), (TF32, 96, 100, 36),
                   (INT8, 130, 260, 272), (FP8, 1, 17, 48), (MXF4, 136, 264, 544),
                   (FP16, 1000, 1000, 1000), (MXF4, 129, 257, 96)]
# CUDA-core GEMMs (IEEE FP32 SIMT, FP64 DMMA): tile multiples, ragged edges, odd K
# (element loads), K shorter than one slab.
GEMM_CC_CASES = [(FP32, 256, 256, 64), (FP32, 200, 130, 37), (FP32, 1, 5, 3),
                 (FP64, 256, 256, 64), (FP64, 130, 200, 37), (FP64, 129, 127, 1000),
                 (FP32, 640, 384, 1024)]


@pytest.mark.parametrize("dtype,m,n,k", GEMM_CASES + GEMM_TAIL_CASES + GEMM_CC_CASES)
def test_gemm_exact(cuda, native, dtype, m, n, k):
    """C = A . B^T through tcb_gemm against the exact host product."""
    a, b = _operands(dtype, 1, 1, m, n, k, seed=m + n + k)
    a, b = a[0], b[0, 0]
    sa = sb = None
    if dtype == MXF4:
        gen = torch.Generator().manual_seed(k)
        sa = torch.randint(125, 130, (m, k // 32), generator=gen, dtype=torch.uint8)
        sb = torch.randint(125, 130, (n, k // 32), generator=gen, dtype=torch.uint8)
    out_dtype = torch.int32 if dtype == INT8 else torch.float64 if dtype == FP64 else torch.float32
    c = torch.full((m, n), -7, dtype=out_dtype, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    psa = psb = None
    if dtype == MXF4:
        psa = torch.empty(native.mx_scales_packed_bytes(m, k // 32), dtype=torch.uint8,
                          device=cuda)
        psb = torch.empty(native.mx_scales_packed_bytes(n, k // 32), dtype=torch.uint8,
                          device=cuda)
        native.mx_scales_pack(sa.to(cuda), psa, m, k // 32)
        native.mx_scales_pack(sb.to(cuda), psb, n, k // 32)
    native.gemm(dtype, a.to(cuda), b.to(cuda), c, m, n, k, scale_a=psa, scale_b=psb,
                status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    if dtype == MXF4:
        ref = oracle_tensor.resident_reference(a.numpy(), b.numpy(), 1, "fp4", sa.numpy(),
                                               sb.numpy())
    else:
        ref = oracle_tensor.resident_reference(_host(a), _host(b), 1, NAME[dtype])
    assert np.array_equal(c.cpu().double().numpy(), ref.astype(np.float64))


@pytest.mark.parametrize("key", ["fp32", "tf32", "fp64"])
def test_gemm_precision_probes(cuda, key):
    """The reference's fp32/tf32/fp64 probes through the GEMM kernels (gemm mode)."""
    from triton_chip_benchmarks_b200 import bench_tensor
    result = bench_tensor.validate_gemm_precision(cuda, key)
    assert result["passed"] and result["kernel_mode"] == "gemm"


def test_gemm_cuda_core_kernel_info(native, cuda):
    fp32 = native.kernel_info(native.FAMILY_GEMM, FP32)
    assert fp32["instruction"] == "fma.rn.f32" and fp32["execution_kind"] == "simt"
    fp64 = native.kernel_info(native.FAMILY_GEMM, FP64)
    assert "m16n8k4" in fp64["instruction"] and fp64["execution_kind"] == "tensor"
    assert fp32["local_bytes_per_thread"] == 0 and fp64["local_bytes_per_thread"] == 0


@pytest.mark.parametrize("dtype,m,n,k", [(INT8, 3400, 3328, 256), (BF16, 3328, 3400, 192),
                                         (FP8, 3584, 3352, 128)])
def test_gemm_256_row_tiles(cuda, native, dtype, m, n, k):
    """Problems with at least as many 256 x 256 tiles as SMs run on the two-accumulator
    kernel (256-row tiles); M tails that are not multiples of 256 are masked."""
    info = native.kernel_info(native.FAMILY_GEMM, dtype, m, n)
    assert (info["tile_m"], info["tile_n"], info["cluster_ctas"]) == (256, 256, 1)
    assert info["pipeline_stages"] >= 2
    a, b = _operands(dtype, 1, 1, m, n, k, seed=m + k)
    a, b = a[0], b[0, 0]
    out_dtype = torch.int32 if dtype == INT8 else torch.float32
    c = torch.full((m, n), -7, dtype=out_dtype, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    native.gemm(dtype, a.to(cuda), b.to(cuda), c, m, n, k, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = oracle_tensor.resident_reference(_host(a), _host(b), 1, NAME[dtype])
    assert np.array_equal(c.cpu().numpy().astype(np.float64), ref.astype(np.float64))


def test_gemm_kernel_info_follows_the_shape(cuda, native):
    """Small problems use 128-row tiles; MX FP4 above 128 rows uses CTA pairs."""
    small = native.kernel_info(native.FAMILY_GEMM, BF16, 1024, 1024)
    assert (small["tile_m"], small["cluster_ctas"]) == (128, 1)
    pair = native.kernel_info(native.FAMILY_GEMM, MXF4, 8192, 8192)
    assert (pair["tile_m"], pair["tile_n"], pair["cluster_ctas"]) == (256, 256, 2)
    assert "cta_group::2" in pair["instruction"]
    single = native.kernel_info(native.FAMILY_GEMM, MXF4, 128, 8192)
    assert (single["tile_m"], single["cluster_ctas"]) == (128, 1)
    assert "cta_group::1" in single["instruction"]


def test_gemm_persistent_tiles(cuda, native):
    """More tiles than CTAs: each CTA walks several tiles through one accumulator."""
    m, n, k = 1024, 1024, 512
    a, b = _operands(BF16, 1, 1, m, n, k, seed=3)
    a, b = a[0], b[0, 0]
    c = torch.zeros((m, n), device=cuda)
    native.gemm(BF16, a.to(cuda), b.to(cuda), c, m, n, k, blocks=5)
    torch.cuda.synchronize()
    ref = oracle_tensor.resident_reference(_host(a), _host(b), 1, "bf16")
    assert np.array_equal(c.cpu().double().numpy(), ref)


def test_gemm_mxf4_pairs_walk_several_tiles(cuda, native):
    """MX FP4 on CTA pairs: 2 pairs walk 16 tiles of 256 x 256, per-group scales."""
    m, n, k = 1024, 1024, 512
    a, b = _operands(MXF4, 1, 1, m, n, k, seed=11)
    a, b = a[0], b[0, 0]
    gen = torch.Generator().manual_seed(12)
    sa = torch.randint(124, 131, (m, k // 32), generator=gen, dtype=torch.uint8)
    sb = torch.randint(124, 131, (n, k // 32), generator=gen, dtype=torch.uint8)
    psa = torch.empty(native.mx_scales_packed_bytes(m, k // 32), dtype=torch.uint8, device=cuda)
    psb = torch.empty(native.mx_scales_packed_bytes(n, k // 32), dtype=torch.uint8, device=cuda)
    native.mx_scales_pack(sa.to(cuda), psa, m, k // 32)
    native.mx_scales_pack(sb.to(cuda), psb, n, k // 32)
    c = torch.full((m, n), -7.0, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    native.gemm(MXF4, a.to(cuda), b.to(cuda), c, m, n, k, scale_a=psa, scale_b=psb, blocks=4,
                status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = oracle_tensor.resident_reference(a.numpy(), b.numpy(), 1, "fp4", sa.numpy(), sb.numpy())
    assert np.array_equal(c.cpu().double().numpy(), ref)


def test_gemm_rejects_unsupported_shapes(cuda, native):
    # K = 60 bf16 elements: a 120-byte row is not a whole number of 16-byte units.
    a = torch.zeros((128, 60), dtype=torch.bfloat16, device=cuda)
    c = torch.zeros((128, 128), device=cuda)
    with pytest.raises(native.TcbError) as info:
        native.gemm(BF16, a, a, c, 128, 128, 60)
    assert info.value.is_capability


@pytest.mark.parametrize("rows,groups", [(128, 8), (256, 64), (768, 256), (130, 17), (1, 1)])
def test_mx_scales_pack_matches_oracle(cuda, native, rows, groups):
    gen = torch.Generator().manual_seed(rows + groups)
    src = torch.randint(0, 256, (rows, groups), generator=gen, dtype=torch.uint8)
    dst = torch.zeros(native.mx_scales_packed_bytes(rows, groups), dtype=torch.uint8,
                      device=cuda)
    native.mx_scales_pack(src.to(cuda), dst, rows, groups)
    torch.cuda.synchronize()
    assert np.array_equal(dst.cpu().numpy(), oracle_tensor.pack_mx_scales(src.numpy()))
