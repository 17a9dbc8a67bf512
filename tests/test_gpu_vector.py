"""Vector FMA-chain kernels through the C ABI, bit-exact against the oracle (GPU)."""

import numpy as np
import pytest
import torch

from oracle import native as oracle_native
from oracle import vector as oracle_vector

pytestmark = pytest.mark.gpu

BF16, FP16, FP32, FP64, DP4A, IMAD, I8 = range(7)


@pytest.fixture(params=["device", "host"])
def coeff_where(request):
    """Coefficients in device memory (tcb_vector_chains) or host memory, passed to
    the kernel by value (tcb_vector_chains_imm)."""
    return request.param


def _run(native, cuda, dtype, inputs, coeff, iterations, blocks, threads, ept, unroll,
         where="device"):
    x = inputs.to(cuda)
    out = torch.empty_like(x)
    native.vector_chains(dtype, x, out, coeff.to(cuda) if where == "device" else coeff.contiguous(),
                         inputs.shape[1], iterations, blocks, threads, ept, unroll)
    torch.cuda.synchronize()
    return out.cpu()


def _float_inputs(kind, elements, seed, baseline):
    gen = torch.Generator().manual_seed(seed)
    dtype = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32,
             "f64": torch.float64}[kind]
    if baseline:
        x = (torch.rand((8, elements), generator=gen, dtype=torch.float64) * 0.5 + 0.5).to(dtype)
        coeff = torch.tensor([0.9990234375] + [0.0009765625] * 8, dtype=dtype)
    elif kind in ("bf16", "f16"):
        x = (torch.randint(1, 8, (8, elements), generator=gen).double() / 8).to(dtype)
        coeff = torch.tensor([-1.0] + [(i + 1) / 8 for i in range(8)], dtype=dtype)
    else:
        x = (torch.rand((8, elements), generator=gen, dtype=torch.float64) * 0.875 + 0.125).to(dtype)
        coeff = torch.tensor([1.0 - 2.0**-14] + [(c + 1) * 2.0**-16 for c in range(8)], dtype=dtype)
    return x, coeff


def _as_bits(t):
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@pytest.mark.parametrize("kind,code", [("f32", FP32), ("f64", FP64), ("f16", FP16),
                                       ("bf16", BF16)])
@pytest.mark.parametrize("baseline", [False, True])
@pytest.mark.parametrize("ept,unroll", [(2, 1), (4, 4), (8, 16), (16, 8)])
@pytest.mark.parametrize("iterations", [1, 33, 256])
def test_float_chains_bit_exact(cuda, native, kind, code, baseline, ept, unroll, iterations,
                                coeff_where):
    if kind == "f64" and ept == 16:
        pytest.skip("fp64 with 16 elements per thread spills; not a swept configuration")
    blocks, threads = 3, 64
    elements = blocks * threads * ept
    x, coeff = _float_inputs(kind, elements, iterations + ept, baseline)
    got = _run(native, cuda, code, x, coeff, iterations, blocks, threads, ept, unroll, coeff_where)
    expected = oracle_native.chain(kind, _as_bits(x), _as_bits(coeff), iterations)
    assert np.array_equal(_as_bits(got), expected)


@pytest.mark.parametrize("ept,unroll", [(1, 1), (4, 8), (16, 16)])
@pytest.mark.parametrize("iterations", [1, 2, 3, 32, 4096])
def test_dp4a_chains_exact(cuda, native, ept, unroll, iterations, coeff_where):
    blocks, threads = 2, 32
    elements = blocks * threads * ept
    gen = torch.Generator().manual_seed(iterations)
    x = torch.randint(-(2**31), 2**31, (8, elements), generator=gen).to(torch.int32)
    coeff = torch.tensor([oracle_vector.packed_dp4a_weights()] + list(range(1, 9)),
                         dtype=torch.int32)
    got = _run(native, cuda, DP4A, x, coeff, iterations, blocks, threads, ept, unroll, coeff_where)
    assert np.array_equal(got.numpy(), oracle_native.chain("dp4a", x.numpy(), coeff.numpy(),
                                                           iterations))
    lifted = oracle_vector.dp4a_reference(x.numpy(), coeff.numpy(), iterations)
    assert np.array_equal(got.numpy().astype(np.int64), lifted)


@pytest.mark.parametrize("a,iterations", [(1, 8192), (3, 33), (-7, 1000)])
def test_imad_chains_exact(cuda, native, a, iterations, coeff_where):
    blocks, threads, ept = 2, 64, 4
    elements = blocks * threads * ept
    gen = torch.Generator().manual_seed(a + iterations)
    x = torch.randint(-(2**31), 2**31, (8, elements), generator=gen).to(torch.int32)
    coeff = torch.tensor([a] + [2 * c + 1 for c in range(8)], dtype=torch.int32)
    got = _run(native, cuda, IMAD, x, coeff, iterations, blocks, threads, ept, 8, coeff_where)
    assert np.array_equal(got.numpy().astype(np.int64),
                          oracle_vector.imad_reference(x.numpy(), coeff.numpy(), iterations))


@pytest.mark.parametrize("iterations", [1, 2, 3, 32, 4096, 4097])
def test_int8_muladd_exact(cuda, native, iterations, coeff_where):
    blocks, threads, ept = 2, 32, 8
    elements = blocks * threads * ept
    gen = torch.Generator().manual_seed(iterations)
    x = torch.randint(-128, 128, (8, elements), generator=gen).to(torch.int8)
    coeff = torch.tensor([3] + [2 * c + 1 for c in range(8)], dtype=torch.int8)
    got = _run(native, cuda, I8, x, coeff, iterations, blocks, threads, ept, 4, coeff_where)
    assert np.array_equal(got.numpy().astype(np.int64),
                          oracle_vector.mod256_reference(x.numpy(), coeff.numpy(), iterations))


def test_vector_rejects_bad_shapes(cuda, native):
    x = torch.zeros((8, 256), device=cuda)
    with pytest.raises(native.TcbError):
        native.vector_chains(FP32, x, x, torch.zeros(9, device=cuda), 256, 4, 1, 128, 3, 1)
    with pytest.raises(native.TcbError):
        native.vector_chains(FP16, x, x, torch.zeros(9, device=cuda), 256, 4, 2, 128, 1, 1)
    with pytest.raises(native.TcbError):
        native.vector_chains(FP32, x, x, torch.zeros(9), 256, 4, 1, 128, 3, 1)
