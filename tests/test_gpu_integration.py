"""The reference-side ctypes stub (tcb_binding.py) against the built library (GPU).

The stub is what a maintainer adds beside the reference's scripts.  Here its
_launch_peak runs tile shapes from the reference's own sweep
(_peak_configs, bench_tensor.py:491-578) on operands laid out the way the
reference's _peak_inputs lays them out (bench_tensor.py:647-672: A
[blocks, M, K], B [chains, blocks, K, N], ternary values / 16), and every
result must equal iterations x (A . B) exactly.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def stub(cuda):
    from triton_chip_benchmarks_b200 import tcb_binding
    return vars(tcb_binding)


# (dtype, dot_input_precision, block_m, block_n, block_k): the reference's IEEE FP32
# tiles (bench_tensor.py:499-503), its FP64 tiles (:497-498) and its NVIDIA set for
# the tcgen05 kinds (:504-511: 64x64, 64x128, 128x64 at K 32, or 64 for 8-bit).
CASES = [(torch.float32, "ieee", 32, 32, 32), (torch.float32, "ieee", 32, 64, 32),
         (torch.float32, "ieee", 64, 32, 32), (torch.float32, "ieee", 64, 64, 32),
         (torch.float64, None, 32, 32, 16), (torch.float64, None, 32, 64, 16),
         (torch.bfloat16, None, 64, 64, 32), (torch.bfloat16, None, 64, 128, 32),
         (torch.bfloat16, None, 128, 64, 32), (torch.float16, None, 64, 128, 32),
         (torch.float32, "tf32", 64, 64, 32), (torch.float32, "tf32", 128, 64, 32),
         (torch.int8, None, 64, 128, 64), (torch.float8_e4m3fn, None, 64, 64, 64)]


@pytest.mark.parametrize("dtype,precision,m,n,k", CASES)
def test_stub_runs_reference_tiles_exactly(stub, cuda, dtype, precision, m, n, k):
    blocks, chains, iterations = 3, 2, 5
    gen = torch.Generator().manual_seed(m * n + k)
    scale = 1 if dtype == torch.int8 else 16  # ternary, / 16 for the float kinds
    a = (torch.randint(-1, 2, (blocks, m, k), generator=gen).double() / scale).to(dtype)
    b = (torch.randint(-1, 2, (chains, blocks, k, n), generator=gen).double() / scale).to(dtype)
    out_dtype = {torch.float64: torch.float64, torch.int8: torch.int32}.get(dtype, torch.float32)
    c = torch.full((chains, blocks, m, n), -7, dtype=out_dtype, device=cuda)
    config = dict(block_m=m, block_n=n, block_k=k, num_warps=4, num_stages=1, chains=chains)
    stub["_launch_peak"](a.to(cuda), b.to(cuda), c, iterations, config,
                         dot_input_precision=precision)
    torch.cuda.synchronize()
    expected = iterations * np.matmul(a.double().numpy()[None], b.double().numpy())
    assert np.array_equal(c.cpu().double().numpy(), expected)


def test_stub_raises_reference_classifiable_rejection(stub, cuda):
    """A tile the library does not provide (32 rows on a tcgen05 kind) is rejected with
    the message the reference's _unsupported_reason accepts (tests/golden/tensor.json,
    status_classification), so the reference's sweep records it and goes on."""
    a = torch.zeros((1, 32, 32), dtype=torch.bfloat16, device=cuda)
    b = torch.zeros((2, 1, 32, 64), dtype=torch.bfloat16, device=cuda)
    c = torch.zeros((2, 1, 32, 64), device=cuda)
    config = dict(block_m=32, block_n=64, block_k=32, num_warps=4, num_stages=1, chains=2)
    with pytest.raises(RuntimeError, match="unsupported matrix format or tile"):
        stub["_launch_peak"](a, b, c, 1, config)


# (dtype, int8 operation, BLOCK_SIZE, num_warps) from the reference's NVIDIA vector
# sweep (BLOCK 256-2048, warps 4 or 8): 256 elements over 8 warps is one element per
# thread, which the stub runs on packed pairs for the 16-bit types.
VECTOR_CASES = [("fp32", "dp4a", 1024, 4), ("fp64", "dp4a", 512, 8), ("bf16", "dp4a", 256, 8),
                ("fp16", "dp4a", 256, 4), ("fp16", "dp4a", 2048, 8), ("int8", "dp4a", 2048, 8),
                ("int8", "muladd", 512, 4)]


@pytest.mark.parametrize("dtype,int8_op,block_size,num_warps", VECTOR_CASES)
def test_stub_launch_vector_called_as_the_reference_calls_it(stub, cuda, dtype, int8_op,
                                                             block_size, num_warps):
    from types import SimpleNamespace

    from triton_chip_benchmarks_b200 import bench_vector
    args = SimpleNamespace(dtype=dtype, inputs="reference", seed=3, int8_op=int8_op)
    blocks, iterations, unroll = 3, 64, 4
    elements = blocks * block_size
    inputs, coeff = bench_vector.make_inputs(args, elements, cuda)
    output = torch.empty_like(inputs)
    is_int8 = dtype == "int8"
    use_dp4a = is_int8 and int8_op == "dp4a"
    # The reference's positional call, bench_vector.py:1411-1416 (kernel object unused).
    stub["launch_vector"](None, (blocks,), inputs, output, coeff, elements, iterations,
                          block_size, unroll, True, num_warps, is_int8, use_dp4a, False, False,
                          False, False)
    torch.cuda.synchronize()
    bench_vector.validate(args, inputs, output, coeff, iterations)  # raises on a mismatch


def test_stub_copy_and_read_called_as_the_reference_calls_them(stub, cuda):
    """launch_copy / launch_read with the reference's arguments (bench_bandwidth.py:
    43-67), on an element count that fills neither a block nor a 16-byte vector."""
    n = 4096 * 3 + 17
    src = torch.randn(n, device=cuda)
    dst = torch.full_like(src, float("nan"))
    stub["launch_copy"](src, dst, 4096, 4)
    block = 1024
    sink = torch.full((-(-n // block),), float("nan"), device=cuda)
    stub["launch_read"](src, sink, block, 8, "nvidia")
    torch.cuda.synchronize()
    assert torch.equal(src, dst)
    expected = torch.nn.functional.pad(src.double(), (0, sink.numel() * block - n))
    expected = expected.view(-1, block).sum(1)
    assert torch.allclose(sink.double(), expected, rtol=1e-5, atol=1e-3)


# (dtype, dot_input_precision, M, N, K) in GEMM mode, operands as the reference's
# _inputs builds them (bench_tensor.py:249-261: randn A, randn B / sqrt(K), ternary
# int8), B [K, N] row-major; tolerances of the reference's _validate (:289-299).
GEMM_CASES = [(torch.bfloat16, None, 256, 256, 256, 2e-3), (torch.float16, None, 192, 320, 64, 2e-3),
              (torch.float32, "tf32", 256, 128, 128, 1e-2), (torch.float32, "ieee", 200, 136, 72, 2e-3),
              (torch.float64, None, 96, 160, 48, 1e-10), (torch.int8, None, 256, 256, 128, 0.0)]


@pytest.mark.parametrize("dtype,precision,m,n,k,tol", GEMM_CASES)
def test_stub_gemm_launch_as_the_reference_calls_it(stub, cuda, dtype, precision, m, n, k, tol):
    gen = torch.Generator().manual_seed(m + n + k)
    if dtype == torch.int8:
        a = torch.randint(-1, 2, (m, k), generator=gen, dtype=dtype)
        b = torch.randint(-1, 2, (k, n), generator=gen, dtype=dtype)
        out_dtype = torch.int32
    else:
        wide = torch.float64 if dtype == torch.float64 else torch.float32
        a = torch.randn((m, k), generator=gen, dtype=wide).to(dtype)
        b = (torch.randn((k, n), generator=gen, dtype=wide) / k ** 0.5).to(dtype)
        out_dtype = torch.float64 if dtype == torch.float64 else torch.float32
    c = torch.empty((m, n), dtype=out_dtype, device=cuda)
    config = dict(block_m=128, block_n=128, block_k=64, num_warps=4, num_stages=3)
    a_dev, b_dev = a.to(cuda), b.to(cuda)
    for _ in range(2):  # the second call uses the stub's cached K-contiguous B
        c.fill_(0)
        stub["_launch"](a_dev, b_dev, c, config, precision)
        torch.cuda.synchronize()
        expected = a.double() @ b.double()
        got = c.cpu().double()
        if tol == 0.0:
            assert torch.equal(got, expected)
        else:
            assert torch.allclose(got, expected, rtol=tol, atol=tol)
