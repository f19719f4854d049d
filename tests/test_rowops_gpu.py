"""RMSNorm, residual RMSNorm, RoPE and SiLU (tests/test_advanced12.py:104-177)
on the GPU through the reference-named launches, against the oracle: RoPE bit
for bit, the rest at atol = rtol = 1e-5 (the reference's own checks allow
1e-3, 1e-3, 1e-4 and 1e-5 absolute, :243-298). Covers the reference's launch
shapes, ragged and strided rows, BLOCK sizes that cover only part of a row
(the columns past BLOCK stay untouched, as in the reference), and in-place
calls."""
import pytest
import torch

import oracle
from neso_b200 import kernels

pytestmark = pytest.mark.gpu
TOL = dict(atol=1e-5, rtol=1e-5)


def _cdiv(a, b):
    return (a + b - 1) // b


def test_reference_launches(dev):
    g = torch.Generator().manual_seed(0)
    M, N, eps = 32, 128, 1e-5
    x, r = torch.randn(M, N, generator=g), torch.randn(M, N, generator=g)
    w = torch.randn(N, generator=g)
    out = torch.zeros(M, N, device=dev)
    kernels.rmsnorm_kernel[(M,)](x.to(dev), w.to(dev), out, N, N, eps, BLOCK_SIZE=128)
    torch.testing.assert_close(out.cpu(), oracle.rmsnorm(x, w, eps), **TOL)
    out = torch.zeros(M, N, device=dev)
    kernels.residual_rmsnorm_kernel[(M,)](x.to(dev), r.to(dev), w.to(dev), out, N, N, eps, BLOCK_SIZE=128)
    torch.testing.assert_close(out.cpu(), oracle.rmsnorm(x, w, eps, residual=r), **TOL)

    n = 2048
    xs = torch.randn(n, generator=g)
    o = torch.zeros(n, device=dev)
    kernels.silu_kernel[lambda m: (_cdiv(n, m["BLOCK"]),)](xs.to(dev), o, n, BLOCK=256)
    torch.testing.assert_close(o.cpu(), oracle.silu(xs), atol=1e-6, rtol=1e-5)

    seq_len, head_dim = 16, 64
    half = head_dim // 2
    xr = torch.randn(seq_len, head_dim, generator=g)
    pos = torch.arange(seq_len).float()
    freq = 1.0 / (10000.0 ** (torch.arange(half).float() / half))
    ang = pos[:, None] * freq[None, :]
    cs, sn = torch.cos(ang), torch.sin(ang)
    out = torch.zeros(seq_len, head_dim, device=dev)
    kernels.rope_kernel[(seq_len,)](xr.to(dev), cs.to(dev), sn.to(dev), out, seq_len, head_dim, BLOCK_D=32)
    a, b = oracle.rope(xr, cs, sn, 32)
    assert torch.equal(out.cpu(), torch.cat([a, b], dim=1))


@pytest.mark.parametrize("residual", [False, True])
def test_rmsnorm_large_strided_partial_and_in_place(dev, residual):
    g = torch.Generator().manual_seed(1 + residual)
    eps = 1e-6
    # 16-byte path: 1000 rows of 4096
    M, N = 1000, 4096
    x, r, w = torch.randn(M, N, generator=g), torch.randn(M, N, generator=g), torch.randn(N, generator=g)
    out = torch.empty(M, N, device=dev)
    args = (x.to(dev), r.to(dev)) if residual else (x.to(dev),)
    k = kernels.residual_rmsnorm_kernel if residual else kernels.rmsnorm_kernel
    k[(M,)](*args, w.to(dev), out, N, N, eps, BLOCK_SIZE=4096)
    torch.testing.assert_close(out.cpu(), oracle.rmsnorm(x, w, eps, residual=r if residual else None), **TOL)
    # scalar path: rows 1001 apart, 1000 columns; column 1000 of every row untouched
    M, N, S = 37, 1000, 1001
    xb, rb = torch.randn(M, S, generator=g), torch.randn(M, S, generator=g)
    w = torch.randn(N, generator=g)
    out = torch.full((M, S), 7.0, device=dev)
    args = (xb.to(dev), rb.to(dev)) if residual else (xb.to(dev),)
    k[(M,)](*args, w.to(dev), out, S, N, eps, BLOCK_SIZE=1024)
    ref = oracle.rmsnorm(xb[:, :N], w, eps, residual=rb[:, :N] if residual else None)
    torch.testing.assert_close(out[:, :N].cpu(), ref, **TOL)
    assert torch.all(out[:, N:] == 7.0)
    # BLOCK_SIZE < n_cols: only the first 128 of 300 columns, mean over 300
    M, N = 9, 300
    x, r, w = torch.randn(M, N, generator=g), torch.randn(M, N, generator=g), torch.randn(N, generator=g)
    out = torch.full((M, N), 7.0, device=dev)
    args = (x.to(dev), r.to(dev)) if residual else (x.to(dev),)
    k[(M,)](*args, w.to(dev), out, N, N, eps, BLOCK_SIZE=128)
    ref = oracle.rmsnorm(x, w, eps, residual=r if residual else None, block=128)
    torch.testing.assert_close(out[:, :128].cpu(), ref, **TOL)
    assert torch.all(out[:, 128:] == 7.0)
    # in place (out is x)
    M, N = 64, 512
    x, r, w = torch.randn(M, N, generator=g), torch.randn(M, N, generator=g), torch.randn(N, generator=g)
    xd = x.to(dev)
    args = (xd, r.to(dev)) if residual else (xd,)
    k[(M,)](*args, w.to(dev), xd, N, N, eps, BLOCK_SIZE=512)
    torch.testing.assert_close(xd.cpu(), oracle.rmsnorm(x, w, eps, residual=r if residual else None), **TOL)


@pytest.mark.parametrize("seq_len,head_dim,block_d", [(1000, 128, 64), (300, 128, 16), (7, 65, 32)])
def test_rope_bit_exact(dev, seq_len, head_dim, block_d):
    # block_d = 16 < head_dim / 2 rotates only the first 16 pairs; head_dim = 65
    # leaves the last column alone (half = 32).
    g = torch.Generator().manual_seed(seq_len)
    half = head_dim // 2
    x = torch.randn(seq_len, head_dim, generator=g)
    cs, sn = torch.randn(seq_len, half, generator=g), torch.randn(seq_len, half, generator=g)
    out = torch.full((seq_len, head_dim), 7.0, device=dev)
    kernels.rope_kernel[(seq_len,)](x.to(dev), cs.to(dev), sn.to(dev), out, seq_len, head_dim, BLOCK_D=block_d)
    a, b = oracle.rope(x, cs, sn, block_d)
    hd = a.shape[1]
    o = out.cpu()
    assert torch.equal(o[:, :hd], a) and torch.equal(o[:, half:half + hd], b)
    untouched = torch.ones(head_dim, dtype=torch.bool)
    untouched[:hd] = False
    untouched[half:half + hd] = False
    assert torch.all(o[:, untouched] == 7.0)
    # in place
    xd = x.to(dev)
    kernels.rope_kernel[(seq_len,)](xd, cs.to(dev), sn.to(dev), xd, seq_len, head_dim, BLOCK_D=block_d)
    assert torch.equal(xd.cpu()[:, :hd], a) and torch.equal(xd.cpu()[:, half:half + hd], b)


def test_silu_ragged_and_unaligned(dev):
    g = torch.Generator().manual_seed(5)
    n = 1_000_003
    x = torch.randn(n + 1, generator=g) * 8
    xd = x.to(dev)
    out = torch.empty(n + 1, device=dev)
    kernels.silu_kernel[(_cdiv(n, 1024),)](xd, out, n, BLOCK=1024)  # 16-byte path + tail
    torch.testing.assert_close(out[:n].cpu(), oracle.silu(x[:n]), atol=1e-6, rtol=1e-5)
    out2 = torch.empty(n + 1, device=dev)
    kernels.silu_kernel[(_cdiv(n, 1024),)](xd[1:], out2[1:], n, BLOCK=1024)  # 4-byte offset: scalar path
    torch.testing.assert_close(out2[1:].cpu(), oracle.silu(x[1:]), atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("M,N,block", [(16, 128, 128), (8, 256, 256), (300, 1000, 1024), (5, 300, 128)])
def test_softmax_rows(dev, M, N, block):
    # tests/test_triton_jit.py:307-325 launches, plus long, strided-output and
    # partial-row (BLOCK_SIZE < n_cols: the columns past BLOCK_SIZE untouched) cases.
    g = torch.Generator().manual_seed(M + N)
    x = torch.randn(M, N, generator=g) * 4
    out = torch.full((M, N + 3), 7.0, device=dev)
    kernels.softmax_kernel[(M,)](out, x.to(dev), N, N + 3, N, BLOCK_SIZE=block)
    c = min(block, N)
    torch.testing.assert_close(out[:, :c].cpu(), oracle.softmax_rows(x, block), atol=1e-6, rtol=1e-5)
    assert torch.all(out[:, c:] == 7.0)


def test_dequant_and_quantize(dev):
    # tests/test_advanced12.py:216-241 launches (int8 values in int32 tensors) plus ragged sizes;
    # quantize follows the kernel's own rounding bit for bit.
    g = torch.Generator().manual_seed(9)
    for (M, N) in [(32, 64), (77, 1001)]:
        x = torch.randint(-128, 127, (M, N), generator=g, dtype=torch.int32)
        sc = torch.rand(N, generator=g) * 0.1 + 0.01
        zr = torch.randint(-5, 5, (N,), generator=g).float()
        out = torch.zeros(M, N, device=dev)
        kernels.per_channel_dequant_kernel[(_cdiv(M, 32), _cdiv(N, 32))](x.to(dev), sc.to(dev), zr.to(dev), out, M, N,
                                                                         BLOCK_M=32, BLOCK_N=32)
        assert torch.equal(out.cpu(), oracle.per_channel_dequant(x, sc, zr))
    for (n, gs) in [(1024, 128), (100_003, 64)]:
        x = torch.randint(-128, 127, (n,), generator=g, dtype=torch.int32)
        ng = _cdiv(n, gs)
        sc = torch.rand(ng, generator=g) * 0.1 + 0.01
        zr = torch.randint(-5, 5, (ng,), generator=g).float()
        out = torch.zeros(n, device=dev)
        kernels.grouped_dequant_kernel[lambda m: (_cdiv(n, m["BLOCK"]),)](x.to(dev), sc.to(dev), zr.to(dev), out, n,
                                                                          gs, BLOCK=256)
        assert torch.equal(out.cpu(), oracle.grouped_dequant(x, sc, zr, gs))
    for n in (1024, 50_001):
        x = torch.randn(n, generator=g) * 10
        x[:4] = torch.tensor([1e6, -1e6, 0.5, -0.5])  # clamping and ties
        scale = torch.tensor([x[4:].abs().max().item() / 127.0])
        out = torch.zeros(n, device=dev, dtype=torch.int32)
        kernels.quantize_kernel[(_cdiv(n, 256),)](x.to(dev), scale.to(dev), out, n, BLOCK=256)
        assert torch.equal(out.cpu(), oracle.quantize_int8(x, scale))
