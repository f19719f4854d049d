"""Dense fp16 GEMM (fp32 C) on the GPU against the oracle, atol = rtol = 2e-3
(tests/test_aot.py:70-99, bench/bench_matmul.py:77-153)."""
import math

import pytest
import torch

import oracle
from neso_b200 import _lib, kernels, ops

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=2e-3)


def _inputs(M, N, K, seed=0):
    # BASELINE: A, B ~ N(0, 1/sqrt(K)) (std), fp16
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(M, K, generator=g) / math.sqrt(K)).half()
    b = (torch.randn(K, N, generator=g) / math.sqrt(K)).half()
    return a, b


@pytest.mark.parametrize("M,N,K", [
    (128, 256, 64),      # one 128x256 tile, one k-block
    (128, 128, 128),
    (256, 64, 64),       # BN = 64 path
    (384, 512, 320),     # several tiles, ragged k-blocks (320 = 5 x 64)
    (1, 256, 64),        # M = 1
    (200, 136, 72),      # ragged M, N and K (TMA zero fill + masked stores)
    (1024, 1024, 1024),  # BASELINE size
])
def test_matmul_vs_oracle(dev, M, N, K):
    a, b = _inputs(M, N, K)
    c = ops.matmul(a.to(dev), b.to(dev))
    ref = oracle.gemm(a, b)
    torch.testing.assert_close(c.cpu(), ref, **TOL)


def test_matmul_2048_and_4096(dev):
    for n in (2048, 4096):
        a, b = _inputs(n, n, n, seed=n)
        c = ops.matmul(a.to(dev), b.to(dev))
        torch.testing.assert_close(c.cpu(), oracle.gemm(a, b), **TOL)


@pytest.mark.parametrize("M,N,K", [
    (4000, 4000, 200),   # 256 x 256 tiles: ragged last row tile, column tile and K block
    (832, 9472, 136),    # 4 x 37 = 148 tiles; the last row tile's second half is entirely past M
])
def test_matmul_256_row_tiles_ragged(dev, M, N, K):
    a, b = _inputs(M, N, K, seed=M)
    c = ops.matmul(a.to(dev), b.to(dev))
    torch.testing.assert_close(c.cpu(), oracle.gemm(a, b), **TOL)


@pytest.mark.parametrize("M,N,K", [
    (1928, 2040, 1000),  # ragged M, N not a multiple of 64 (2-D B copies), ragged K; C blocks past N skipped
    (2048, 2048, 64),    # one K block per tile
    (2304, 4352, 520),   # several tiles per CTA, both accumulators in use
    (2048, 2080, 128),   # 128 x 256 tiles: the last column tile stores one 32-column block and skips seven
])
def test_matmul_ragged_large(dev, M, N, K):
    a, b = _inputs(M, N, K, seed=M + N)
    c = ops.matmul(a.to(dev), b.to(dev))
    torch.testing.assert_close(c.cpu(), oracle.gemm(a, b), **TOL)


def test_matmul_unaligned_c_large(dev):
    # C row stride of N + 3 floats: the epilogue writes rows with plain stores
    M, N, K = 2048, 2048, 256
    a, b = _inputs(M, N, K, seed=11)
    c = torch.zeros(M, N + 3, device=dev)
    kernels.matmul_kernel[(M // 128, N // 128, 1)](a.to(dev), b.to(dev), c, M, N, K, K, 1, N, 1, N + 3, 1,
                                                   BLOCK_M=128, BLOCK_N=128, BLOCK_K=64)
    torch.testing.assert_close(c[:, :N].cpu(), oracle.gemm(a, b), **TOL)


def test_matmul_8192_sampled(dev):
    # Full BASELINE size; compare a sample of rows against the oracle.
    n = 8192
    g = torch.Generator(device=dev).manual_seed(1)
    a = (torch.randn(n, n, device=dev, generator=g) / math.sqrt(n)).half()
    b = (torch.randn(n, n, device=dev, generator=g) / math.sqrt(n)).half()
    c = ops.matmul(a, b)
    rows = torch.tensor([0, 1, 127, 128, 4095, 8191])
    ref = oracle.gemm(a[rows.to(dev)].cpu(), b.cpu())
    torch.testing.assert_close(c[rows.to(dev)].cpu(), ref, **TOL)


def test_reference_style_launch_with_strides(dev):
    # matmul_kernel[grid](a, b, c, M, N, K, strides..., BLOCK_M, BLOCK_N, BLOCK_K) (tests/test_aot.py:197-202)
    M, N, K = 256, 192, 96
    a, b = _inputs(M, N, K, seed=5)
    big = torch.zeros(M, K + 8, dtype=torch.float16)
    big[:, :K] = a
    ad, bd = big.to(dev), b.to(dev)
    c = torch.zeros(M, N + 4, device=dev)
    grid = lambda meta: ((meta["M"] + meta["BLOCK_M"] - 1) // meta["BLOCK_M"],
                         (meta["N"] + meta["BLOCK_N"] - 1) // meta["BLOCK_N"], 1)
    kernels.matmul_kernel[grid](ad, bd, c, M, N, K, K + 8, 1, N, 1, N + 4, 1, BLOCK_M=128, BLOCK_N=64,
                                BLOCK_K=32)
    torch.testing.assert_close(c[:, :N].cpu(), oracle.gemm(a, b), **TOL)
    assert torch.all(c[:, N:] == 0)


def test_c_row_stride_not_multiple_of_4_uses_row_stores(dev):
    # stride_cm = N + 1 floats: C rows are not 16-byte aligned, so the
    # epilogue cannot use TMA stores and writes rows directly.
    M, N, K = 384, 512, 256
    a, b = _inputs(M, N, K, seed=13)
    c = torch.full((M, N + 1), 5.0, device=dev)
    grid = lambda meta: ((meta["M"] + meta["BLOCK_M"] - 1) // meta["BLOCK_M"],
                         (meta["N"] + meta["BLOCK_N"] - 1) // meta["BLOCK_N"], 1)
    kernels.matmul_kernel[grid](a.to(dev), b.to(dev), c, M, N, K, K, 1, N, 1, N + 1, 1, BLOCK_M=128, BLOCK_N=64,
                                BLOCK_K=32)
    torch.testing.assert_close(c[:, :N].cpu(), oracle.gemm(a, b), **TOL)
    assert torch.all(c[:, N:] == 5.0)


def test_matmul_tiled_reference_signature(dev):
    # bench/bench_matmul.py:79-81: matmul_kernel(a, b, c, K, stride_am, stride_bk, stride_cm), grid (M/BM, N/BN)
    M, N, K = 256, 256, 128
    a, b = _inputs(M, N, K, seed=9)
    c = torch.empty(M, N, device=dev)
    kernels.matmul_tiled[(M // 64, N // 32, 1)](a.to(dev), b.to(dev), c, K, K, N, N, BM=64, BN=32)
    torch.testing.assert_close(c.cpu(), oracle.gemm(a, b), **TOL)


def test_zero_k(dev):
    a = torch.zeros(64, 0, dtype=torch.float16, device=dev)
    b = torch.zeros(0, 64, dtype=torch.float16, device=dev)
    c = torch.full((64, 64), 7.0, device=dev)
    kernels.matmul_kernel[(1, 1, 1)](a, b, c, 64, 64, 0, 8, 1, 64, 1, 64, 1)
    assert torch.all(c == 0)


def test_unaligned_stride_rejected(dev):
    a = torch.zeros(64, 70, dtype=torch.float16, device=dev)
    b = torch.zeros(70, 64, dtype=torch.float16, device=dev)
    c = torch.zeros(64, 64, device=dev)
    with pytest.raises(_lib.NesoError) as ei:
        kernels.matmul_kernel[(1, 1, 1)](a, b, c, 64, 64, 70, 70, 1, 64, 1, 64, 1)
    assert ei.value.code == _lib.NESO_ERR_MISALIGNED
