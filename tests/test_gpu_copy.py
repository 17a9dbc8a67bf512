"""Copy and read kernels through the C ABI against the CPU oracle (GPU)."""

import numpy as np
import pytest
import torch

from oracle import native as oracle_native

pytestmark = pytest.mark.gpu

SIZES = [1, 15, 16, 17, 4096 + 3, (1 << 20) + 5, (64 << 20) + 3]


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("nbytes", SIZES)
def test_copy_bit_exact(cuda, native, variant, nbytes):
    gen = torch.Generator().manual_seed(nbytes)
    src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, generator=gen).to(cuda)
    dst = torch.zeros(nbytes + 64, dtype=torch.uint8, device=cuda)
    native.copy(src, dst, nbytes, variant)
    torch.cuda.synchronize()
    assert torch.equal(dst[:nbytes], src)
    assert int(dst[nbytes:].count_nonzero()) == 0, "copy wrote past the end"


@pytest.mark.parametrize("offset", [1, 3, 8])
def test_copy_misaligned_falls_back(cuda, native, offset):
    gen = torch.Generator().manual_seed(offset)
    base = torch.randint(0, 256, (1 << 16,), dtype=torch.uint8, generator=gen).to(cuda)
    out = torch.zeros_like(base)
    n = (1 << 16) - 2 * offset
    native.copy(base[offset:], out[offset:], n)
    torch.cuda.synchronize()
    assert torch.equal(out[offset:offset + n], base[offset:offset + n])


@pytest.mark.parametrize("threads,blocks", [(256, 0), (768, 0), (1024, 0), (768, 7), (96, 1)])
def test_copy_thread_configs(cuda, native, threads, blocks):
    """One CTA per piece (blocks 0) and grid-stride grids, with a ragged piece and tail."""
    n = (32 << 20) + 16 * 7 + 5
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device=cuda)
    dst = torch.zeros_like(src)
    native.copy(src, dst, n, native.COPY_LDG128, blocks, threads)
    torch.cuda.synchronize()
    assert torch.equal(src, dst)


@pytest.mark.parametrize("offset,extra", [(0, 16), (16, 0), (16, 48), (32, 8), (0, 15)])
def test_copy_piece_alignment(cuda, native, offset, extra):
    """256-bit vectors (both pointers 32-byte aligned), two 16-byte vectors
    (16-byte aligned), an odd count of 16-byte vectors and a byte tail; bytes
    outside the range stay untouched."""
    n = (8 << 20) + 768 * 32 * 3 + extra
    gen = torch.Generator().manual_seed(offset + extra)
    base = torch.randint(0, 256, (n + 128,), dtype=torch.uint8, generator=gen).to(cuda)
    out = torch.zeros_like(base)
    native.copy(base[offset:], out[offset:], n)
    torch.cuda.synchronize()
    assert torch.equal(out[offset:offset + n], base[offset:offset + n])
    assert int(out[:offset].count_nonzero()) == 0 and int(out[offset + n:].count_nonzero()) == 0


def test_copy_matches_oracle_copy(cuda, native):
    rng = np.random.default_rng(7)
    host = rng.integers(0, 256, size=(8 << 20) + 9, dtype=np.uint8)
    expected = np.empty_like(host)
    oracle_native.copy(host, expected, 4)
    src = torch.from_numpy(host).to(cuda)
    dst = torch.empty_like(src)
    native.copy(src, dst, host.size, native.COPY_BULK)
    torch.cuda.synchronize()
    assert np.array_equal(dst.cpu().numpy(), expected)


@pytest.mark.parametrize("dtype,code", [(torch.float32, 0), (torch.float16, 1),
                                        (torch.bfloat16, 2)])
@pytest.mark.parametrize("block,threads", [(1024, 256), (16384, 256), (16384, 1024)])
def test_read_block_sums(cuda, native, dtype, code, block, threads):
    """Whole blocks of 1-8 vectors per thread take the batched loads, others
    (and the partial last block) the loop; both against the oracle."""
    n = 3 * block * 7 + 17  # partial last block
    gen = torch.Generator().manual_seed(block)
    host = torch.randn(n, generator=gen).to(dtype)
    src = host.to(cuda)
    sink = torch.full((-(-n // block),), float("nan"), device=cuda)
    native.read(src, code, n, sink, block, threads)
    torch.cuda.synchronize()
    sums, abs_sums = oracle_native.block_sums(host.float().numpy(), block)
    tol = abs_sums * 2 * np.finfo(np.float32).eps * max(1, np.log2(block)) + 1e-6
    got = sink.cpu().double().numpy()
    assert np.all(np.abs(got - sums) <= tol)


def test_invalid_arguments_rejected(cuda, native):
    src = torch.zeros(1024, dtype=torch.uint8, device=cuda)
    with pytest.raises(native.TcbError) as info:
        native.copy(src, src, 1024, 7)
    assert info.value.status == native.ERR_INVALID_ARGUMENT
    with pytest.raises(native.TcbError):
        native.read(src, 0, 256, torch.zeros(1, device=cuda), 300)
