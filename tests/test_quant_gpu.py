"""Dequant-fused quantized matmul on the GPU against the oracle (atol = rtol =
2e-3, fp32 output) and the reference's golden vectors at its own criterion
(max_err / max|ref| < 1 %, tests/test_quantized_matmul.py:356-359)."""
import numpy as np
import pytest
import torch

import oracle
from neso_b200 import _lib, kernels, ops

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=2e-3)


def _assert_unscaled(y, x, w):
    # Without a scale the int8 products reach |y| ~ 1e3-1e4, where fp32 sums
    # of K terms in different orders differ in absolute terms in proportion to
    # the partial sums' size; the check is against a float64 sum with
    # atol = 2e-3 + 4e-6 max|y| (the scaled results use plain 2e-3).
    exact = oracle.w8a16_matmul_f64(x, w)
    torch.testing.assert_close(y.cpu().double(), exact, atol=2e-3 + 4e-6 * exact.abs().max().item(), rtol=2e-3)


def _w8(M, N, K, seed=0):
    # BASELINE: X ~ N(0,1) fp16, W int8 uniform [-127, 127], scale U[0.001, 0.02] fp16
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).half()
    w = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int8)
    s = (torch.rand(N, generator=g) * 0.019 + 0.001).half()
    return x, w, s


def _w4(M, N, K, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).half()
    q = torch.randint(-8, 8, (K, N), generator=g, dtype=torch.int8)
    s = (torch.rand(K // 128, N, generator=g) * 0.019 + 0.001).half()
    return x, q, s


@pytest.mark.parametrize("name,seed_kind", [("w8a16_64", "plain"), ("w4a16_64", "plain"),
                                            ("w8a16_scaled_64", "scaled")])
def test_reference_golden(dev, golden_dir, name, seed_kind):
    g = dict(np.load(golden_dir / f"{name}.npz"))
    M, N, K = int(g["M"]), int(g["N"]), int(g["K"])
    a = torch.from_numpy(g["a"]).half()
    b = torch.from_numpy(g["b"])
    c = torch.empty(M, N, device=dev)
    if "scale" in g:
        s = torch.from_numpy(g["scale"]).half()
        # reference launch: grid (cdiv(M, BM), cdiv(N, BN), 1) (tests/test_quantized_matmul.py:433-438)
        kernels.w8a16_scaled_matmul[(M // 32, N // 32, 1)](a.to(dev), b.to(dev), c, s.to(dev), K, K, N, N,
                                                           BM=32, BN=32, BK=32)
    else:
        s = None
        kernels.w8a16_matmul[(M // 32, N // 64, 1)](a.to(dev), b.to(dev), c, K, K, N, N, BM=32, BN=64, BK=32)
    out = c.cpu().numpy()
    rel = np.abs(out - g["ref"]).max() / np.abs(g["ref"]).max()
    assert rel < 0.01  # the reference's own criterion
    torch.testing.assert_close(c.cpu(), oracle.w8a16_matmul(a, b, s), **TOL)


@pytest.mark.parametrize("M", [1, 5, 16, 17, 32, 64, 65, 128, 300])
def test_w8a16_scaled_sizes(dev, M):
    N, K = 384, 512
    x, w, s = _w8(M, N, K, seed=M)
    y = ops.w8a16_matmul(x.to(dev), w.to(dev), s.to(dev))
    torch.testing.assert_close(y.cpu(), oracle.w8a16_matmul(x, w, s), **TOL)
    y2 = ops.w8a16_matmul(x.to(dev), w.to(dev))
    _assert_unscaled(y2, x, w)


@pytest.mark.parametrize("M", [1, 16, 128, 2048])
def test_w8a16_baseline_shapes(dev, M):
    # BASELINE: K = 4096, N = 11008 (ragged last n-tile: 11008 = 86 x 128)
    N, K = 11008, 4096
    x, w, s = _w8(M, N, K, seed=100 + M)
    y = ops.w8a16_matmul(x.to(dev), w.to(dev), s.to(dev))
    if M > 128:
        rows = torch.tensor([0, 1, 255, 1024, M - 1])
        torch.testing.assert_close(y[rows.to(dev)].cpu(), oracle.w8a16_matmul(x[rows], w, s), **TOL)
    else:
        torch.testing.assert_close(y.cpu(), oracle.w8a16_matmul(x, w, s), **TOL)


@pytest.mark.parametrize("M", [1, 3, 16, 40, 64, 65, 100, 128, 129])
def test_w4a16_sizes(dev, M):
    N, K = 256, 384
    x, q, s = _w4(M, N, K, seed=M)
    wq = oracle.pack_int4(q)
    y = ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))
    torch.testing.assert_close(y.cpu(), oracle.w4a16_g128_matmul(x, wq, s), **TOL)


@pytest.mark.parametrize("M", [1, 16, 128, 2048])
def test_w4a16_baseline_shapes(dev, M):
    N, K = 11008, 4096
    x, q, s = _w4(M, N, K, seed=200 + M)
    wq = oracle.pack_int4(q)
    y = ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))
    if M > 128:
        rows = torch.tensor([0, 7, 500, M - 1])
        torch.testing.assert_close(y[rows.to(dev)].cpu(), oracle.w4a16_g128_matmul(x[rows], wq, s), **TOL)
    else:
        torch.testing.assert_close(y.cpu(), oracle.w4a16_g128_matmul(x, wq, s), **TOL)


@pytest.mark.parametrize("kind", ["w8", "w4"])
def test_paired_channel_tiles_ragged(dev, kind):
    # 25 row blocks x 4 channel pairs = 100 paired units (one wave) against
    # 200 single ones (two waves): the 256-channel unit layout runs, with the
    # second tile of the last pair only partly inside N = 1008.
    M, N, K = 3100, 1008, 256
    if kind == "w8":
        x, w, s = _w8(M, N, K, seed=7)
        y = ops.w8a16_matmul(x.to(dev), w.to(dev), s.to(dev))
        ref = oracle.w8a16_matmul(x, w, s)
    else:
        x, q, s = _w4(M, N, K, seed=8)
        wq = oracle.pack_int4(q)
        y = ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))
        ref = oracle.w4a16_g128_matmul(x, wq, s)
    torch.testing.assert_close(y.cpu(), ref, **TOL)


@pytest.mark.parametrize("kind", ["w8", "w4"])
def test_small_m_paired_channel_tiles_ragged(dev, kind):
    # M <= 16 (swapped layout) with 256-channel units: N = 400 leaves the last
    # unit's second tile partly outside N; K ragged for int8.
    M, N = 12, 400
    if kind == "w8":
        K = 1000
        x, w, s = _w8(M, N, K, seed=31)
        y = ops.w8a16_matmul(x.to(dev), w.to(dev), s.to(dev))
        ref = oracle.w8a16_matmul(x, w, s)
    else:
        K = 1152
        x, q, s = _w4(M, N, K, seed=32)
        wq = oracle.pack_int4(q)
        y = ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))
        ref = oracle.w4a16_g128_matmul(x, wq, s)
    torch.testing.assert_close(y.cpu(), ref, **TOL)


def test_w8a16_256_row_units_ragged(dev):
    # 5 row blocks of 256 x 29 channel pairs = 145 units (one wave; 128-row
    # pairs would take two): the two-accumulator layout runs, its last row
    # block holding 76 rows (second 128-row half empty) and K = 3 blocks.
    M, N, K = 1100, 7424, 192
    x, w, s = _w8(M, N, K, seed=11)
    y = ops.w8a16_matmul(x.to(dev), w.to(dev), s.to(dev))
    torch.testing.assert_close(y.cpu(), oracle.w8a16_matmul(x, w, s), **TOL)


def test_w4a16_256_row_units_ragged(dev):
    # 5 row blocks of 256 x 17 channel tiles = 85 units (one wave; 128-row
    # units would take two): the two-accumulator W4A16 layout, last row
    # block holding 76 rows, two quantisation groups along K.
    M, N, K = 1100, 2176, 256
    x, q, s = _w4(M, N, K, seed=12)
    wq = oracle.pack_int4(q)
    y = ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))
    torch.testing.assert_close(y.cpu(), oracle.w4a16_g128_matmul(x, wq, s), **TOL)


@pytest.mark.parametrize("M,N,K", [(200, 256, 1024), (300, 384, 4096), (2048, 1376, 4096)])
def test_w4a16_large_m_carries_the_product_remainder(dev, M, N, K):
    # M >= 129 layout: each weight q * s enters as fp16(q * s) plus the exact
    # remainder (at most 3 significant bits, E5M2 once scaled by 2^8) times
    # an E5M2 copy of X. Against the float64 sum of x * q * s the error must
    # stay well below both the 2e-3 tolerance and the error of fp16(q * s)
    # alone, which shows the remainder term is applied.
    x, q, s = _w4(M, N, K, seed=M + N)
    wq = oracle.pack_int4(q)
    y = ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))
    rows = torch.arange(M) if M <= 300 else torch.tensor([0, 1, 511, 1024, 1500, M - 1])
    srep = s.repeat_interleave(128, dim=0)
    exact = x[rows].double() @ (q.double() * srep.double())
    hi_only = x[rows].double() @ (q.half() * srep).double()
    err = (y[rows.to(dev)].cpu().double() - exact).abs().max().item()
    err_hi = (hi_only - exact).abs().max().item()
    assert err < 5e-4, err
    assert err < err_hi / 4, (err, err_hi)


def test_w8a16_c_row_stride_not_multiple_of_4(dev):
    # Reference launch with stride_cm = N + 1: Y rows are not 16-byte aligned,
    # so the M >= 65 epilogue writes rows directly instead of TMA stores.
    M, N, K = 256, 384, 256
    x, w, s = _w8(M, N, K, seed=21)
    c = torch.full((M, N + 1), 3.0, device=dev)
    kernels.w8a16_scaled_matmul[(M // 64, N // 64, 1)](x.to(dev), w.to(dev), c, s.to(dev), K, K, N, N + 1,
                                                       BM=64, BN=64, BK=32)
    torch.testing.assert_close(c[:, :N].cpu(), oracle.w8a16_matmul(x, w, s), **TOL)
    assert torch.all(c[:, N:] == 3.0)


def test_product_pack_matches_oracle_layout(dev):
    q = torch.randint(-8, 8, (256, 64), dtype=torch.int8)
    assert torch.equal(ops.pack_int4(q), oracle.pack_int4(q))


def test_int4_k_not_multiple_of_128_rejected(dev):
    x = torch.zeros(4, 192, dtype=torch.float16, device=dev)
    wq = torch.zeros(96, 64, dtype=torch.uint8, device=dev)
    s = torch.zeros(2, 64, dtype=torch.float16, device=dev)
    with pytest.raises(_lib.NesoError) as ei:
        ops.w4a16_g128_matmul(x, wq, s)
    assert ei.value.code == _lib.NESO_ERR_UNSUPPORTED


def test_w8a16_tensor_scale_reference_case_int32_weights(dev):
    # tests/test_advanced12.py:182-197: M = N = K = 32, b drawn with
    # randint(-128, 127) and held in int32, scale 0.01 (fp32), grid (1, 1),
    # BLOCK_M = BLOCK_N = BLOCK_K = 32; the reference accepts max error < 0.5.
    M = N = K = 32
    g = torch.Generator().manual_seed(0)
    a = torch.randn(M, K, generator=g).half()
    b = torch.randint(-128, 127, (K, N), generator=g, dtype=torch.int32)
    scale = torch.tensor([0.01], dtype=torch.float32)
    c = torch.zeros(M, N, device=dev)
    kernels.w8a16_matmul_kernel[(1, 1)](a.to(dev), b.to(dev), c, scale.to(dev), M, N, K, K, 1, N, 1, N, 1,
                                        BLOCK_M=32, BLOCK_N=32, BLOCK_K=32)
    ref = oracle.w8a16_matmul_tensor_scale(a, b, 0.01)
    assert (c.cpu() - ref).abs().max().item() < 0.5
    torch.testing.assert_close(c.cpu(), ref, **TOL)


@pytest.mark.parametrize("M", [1, 4, 16, 64, 128, 2048])
@pytest.mark.parametrize("wdtype", [torch.int8, torch.int32])
def test_w8a16_tensor_scale_baseline_shapes(dev, M, wdtype):
    # BASELINE weight shape (K = 4096, N = 11008): the GEMV (M <= 4), the
    # swapped small-M layout with split-K, and the M >= 65 layouts, all with the
    # one fp32 scale applied in the epilogue (or the split-K reduce).
    N, K = 11008, 4096
    x, w, _ = _w8(M, N, K, seed=300 + M)
    s = 0.0137
    c = torch.empty(M, N, device=dev)
    grid = ((M + 63) // 64, (N + 127) // 128)
    kernels.w8a16_matmul_kernel[grid](x.to(dev), w.to(wdtype).to(dev), c, torch.tensor([s], device=dev), M, N, K,
                                      K, 1, N, 1, N, 1, BLOCK_M=64, BLOCK_N=128, BLOCK_K=64)
    torch.testing.assert_close(c.cpu(), oracle.w8a16_matmul_tensor_scale(x, w, s), **TOL)


def test_w8a16_tensor_scale_checks_grid_and_strides(dev):
    z = torch.zeros(64, device=dev)
    with pytest.raises(_lib.NesoError) as ei:
        kernels.w8a16_matmul_kernel[(2, 1)](z, z, z, z, 32, 32, 32, 32, 1, 32, 1, 32, 1,
                                            BLOCK_M=32, BLOCK_N=32, BLOCK_K=32)
    assert ei.value.code == _lib.NESO_ERR_GRID
    with pytest.raises(_lib.NesoError) as ei:
        kernels.w8a16_matmul_kernel[(1, 1)](z, z, z, z, 32, 32, 32, 32, 2, 32, 1, 32, 1,
                                            BLOCK_M=32, BLOCK_N=32, BLOCK_K=32)
    assert ei.value.code == _lib.NESO_ERR_UNSUPPORTED


@pytest.mark.parametrize("kind,M", [("w8", 5), ("w8", 16), ("w8", 40), ("w4", 16), ("w4", 64)])
def test_swapped_split_k_sum_in_kernel_is_repeatable(dev, kind, M):
    # Decode batches (M <= 64) at the BASELINE weight shape split K across
    # CTAs; the last split of each channel group adds the partial sums in
    # split order inside the kernel. Two launches give identical bits and the
    # oracle's result.
    N, K = 11008, 4096
    if kind == "w8":
        x, w, s = _w8(M, N, K, seed=500 + M)
        run = lambda: ops.w8a16_matmul(x.to(dev), w.to(dev), s.to(dev))  # noqa: E731
        expect = oracle.w8a16_matmul(x, w, s)
    else:
        x, q, s = _w4(M, N, K, seed=600 + M)
        wq = oracle.pack_int4(q)
        run = lambda: ops.w4a16_g128_matmul(x.to(dev), wq.to(dev), s.to(dev))  # noqa: E731
        expect = oracle.w4a16_g128_matmul(x, wq, s)
    y1, y2 = run().cpu(), run().cpu()
    assert torch.equal(y1, y2)
    torch.testing.assert_close(y1, expect, **TOL)
