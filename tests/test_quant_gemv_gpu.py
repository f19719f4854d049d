"""Small-M (decode) paths of the quantized matmul that W8A16 with M <= 4 and
W4A16 with M <= 2 take: the TMA-fed streaming kernel (all of X in shared
memory as fp32, so M x K <= 16384) and, for longer K, the K-sliced CUDA-core
GEMV. Checked against the oracle (atol = rtol = 2e-3), their fixed-order
(bit-reproducible) cross-CTA sums, and the shapes and alignments that send a
call to another kernel."""
import pytest
import torch

import oracle
from neso_b200 import _lib, ops

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=2e-3)


def _assert_unscaled(y, x, w):
    # Without a scale the int8 products reach |y| ~ 1e3-1e4, where fp32 sums
    # of K terms in different orders differ in absolute terms in proportion to
    # the partial sums' size; the check is against a float64 sum with
    # atol = 2e-3 + 4e-6 max|y| (the scaled results use plain 2e-3).
    exact = oracle.w8a16_matmul_f64(x, w)
    torch.testing.assert_close(y.cpu().double(), exact, atol=2e-3 + 4e-6 * exact.abs().max().item(), rtol=2e-3)


def _w8(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).half()
    w = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int8)
    s = (torch.rand(N, generator=g) * 0.019 + 0.001).half()
    return x, w, s


def _w4(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).half()
    q = torch.randint(-8, 8, (K, N), generator=g, dtype=torch.int8)
    s = (torch.rand(K // 128, N, generator=g) * 0.019 + 0.001).half()
    return x, oracle.pack_int4(q), s


@pytest.mark.parametrize("M", [1, 2, 3, 4])
@pytest.mark.parametrize("N,K", [(11008, 4096), (400, 1000), (512, 64), (4096, 8192)])
def test_w8a16_small_m(dev, M, N, K):
    # N = 400: partial last 512-channel block; K = 1000: ragged last slice and batch
    x, w, s = _w8(M, N, K, seed=M * 7 + N + K)
    y = ops.w8a16_matmul(x.to(dev), w.to(dev), s.to(dev))
    torch.testing.assert_close(y.cpu(), oracle.w8a16_matmul(x, w, s), **TOL)
    y0 = ops.w8a16_matmul(x.to(dev), w.to(dev))  # unscaled entry
    _assert_unscaled(y0, x, w)


@pytest.mark.parametrize("M", [1, 2])
@pytest.mark.parametrize("N,K", [(11008, 4096), (400, 1152), (256, 128)])
def test_w4a16_small_m(dev, M, N, K):
    x, wq, s = _w4(M, N, K, seed=M * 11 + N + K)
    y = ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))
    torch.testing.assert_close(y.cpu(), oracle.w4a16_g128_matmul(x, wq, s), **TOL)


@pytest.mark.parametrize("kind,M,K", [("w8", 4, 16384), ("w4", 2, 32768)])
def test_long_k_small_m_falls_back_to_tensor_cores(dev, kind, M, K):
    # Few channel blocks and a long K make each CTA's slice of X too large to
    # stage in shared memory; the call must still succeed (tensor-core path).
    N = 11008
    if kind == "w8":
        x, w, s = _w8(M, N, K, seed=K + M)
        y = ops.w8a16_matmul(x.to(dev), w.to(dev), s.to(dev))
        ref = oracle.w8a16_matmul(x, w, s)
    else:
        x, wq, s = _w4(M, N, K, seed=K + M)
        y = ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))
        ref = oracle.w4a16_g128_matmul(x, wq, s)
    torch.testing.assert_close(y.cpu(), ref, **TOL)


def test_small_m_is_bit_reproducible(dev):
    # The K slices are added in a fixed order by the last CTA of each block.
    x, w, s = _w8(1, 11008, 4096, seed=5)
    xd, wd, sd = x.to(dev), w.to(dev), s.to(dev)
    a = ops.w8a16_matmul(xd, wd, sd)
    for _ in range(3):
        assert torch.equal(ops.w8a16_matmul(xd, wd, sd), a)
    x4, wq, s4 = _w4(2, 11008, 4096, seed=6)
    b = ops.w4a16_g128_matmul(x4.to(dev), wq.to(dev), s4.to(dev))
    assert torch.equal(ops.w4a16_g128_matmul(x4.to(dev), wq.to(dev), s4.to(dev)), b)


def test_gemv_and_tensor_core_paths_agree(dev):
    # M = 4 runs the GEMV, M = 5 the tensor-core kernel: the first four rows
    # of the M = 5 product equal the M = 4 product to tolerance.
    x, w, s = _w8(5, 400, 1000, seed=9)
    wd, sd = w.to(dev), s.to(dev)
    y5 = ops.w8a16_matmul(x.to(dev), wd, sd)
    y4 = ops.w8a16_matmul(x[:4].contiguous().to(dev), wd, sd)
    torch.testing.assert_close(y4, y5[:4], **TOL)
    torch.testing.assert_close(y5.cpu(), oracle.w8a16_matmul(x, w, s), **TOL)


def test_int4_scales_must_be_16_byte_aligned(dev):
    # Both paths read the int4 scale table in 16-byte units (vector loads /
    # TMA): a table starting 2 bytes into an allocation is refused, not read.
    x4, wq, s4 = _w4(1, 256, 256, seed=10)
    buf = torch.empty(s4.numel() + 1, dtype=torch.float16, device=dev)
    s_off = buf[1:].view(s4.shape)
    s_off.copy_(s4.to(dev))
    with pytest.raises(_lib.NesoError) as ei:
        ops.w4a16_g128_matmul(x4.to(dev), wq.to(dev), s_off)
    assert ei.value.code == _lib.NESO_ERR_MISALIGNED
