"""The per-GPU problems that a sharded run at 2, 4 and 8 GPUs hands each rank,
checked on one GPU against the oracle (atol = rtol = 2e-3, fp32 output).

A rank of the multi-GPU bench computes its slice as an ordinary launch:
GEMM and quantized matmul over a 16-aligned group of output columns
(N = 11008 gives 5504 / 2752 / 1376 columns, none a multiple of 128;
M = N = K = m gives m / 2, m / 4, m / 8), FA2 over a contiguous range of
the flattened batch x heads. These are the shapes that range of runs reaches
and the single-GPU tests do not, so every rank's slice is pinned here with
the same column and head split the bench takes (neso_b200.shard)."""
import math

import pytest
import torch

import oracle
from neso_b200 import ops, shard

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=2e-3)
QK, QN = 4096, 11008


def _rows(M):
    return torch.tensor(sorted({0, 1, M // 2, M - 1}))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("kind", ["w8", "w4"])
def test_quant_column_shards(dev, world, kind):
    nc = shard.shard_columns(QN, world, world - 1, 16).size
    assert nc * world == QN
    g = torch.Generator().manual_seed(world * 10 + (kind == "w4"))
    if kind == "w8":
        w = torch.randint(-127, 128, (QK, nc), generator=g, dtype=torch.int8)
        s = (torch.rand(nc, generator=g) * 0.019 + 0.001).half()
        wd, sd = w.to(dev), s.to(dev)
    else:
        q = torch.randint(-8, 8, (QK, nc), generator=g, dtype=torch.int8)
        s = (torch.rand(QK // 128, nc, generator=g) * 0.019 + 0.001).half()
        w = oracle.pack_int4(q)
        wd, sd = w.to(dev), s.to(dev)
    for M in (1, 16, 128, 2048):
        x = torch.randn(M, QK, generator=g).half()
        if kind == "w8":
            y = ops.w8a16_matmul(x.to(dev), wd, sd)
        else:
            y = ops.w4a16_g128_matmul(x.to(dev), wd, sd)
        rows = _rows(M) if M > 128 else torch.arange(M)
        ref = oracle.w8a16_matmul(x[rows], w, s) if kind == "w8" else oracle.w4a16_g128_matmul(x[rows], w, s)
        torch.testing.assert_close(y[rows.to(dev)].cpu(), ref, **TOL)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gemm_column_shards(dev, world):
    for m in (1024, 2048, 4096, 8192):
        sh = shard.shard_columns(m, world, world - 1, 16)
        g = torch.Generator().manual_seed(m + world)
        a = (torch.randn(m, m, generator=g) / math.sqrt(m)).half()
        b = (torch.randn(m, sh.size, generator=g) / math.sqrt(m)).half()
        c = ops.matmul(a.to(dev), b.to(dev))
        rows = _rows(m)
        torch.testing.assert_close(c[rows.to(dev)].cpu(), oracle.gemm(a[rows], b), **TOL)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("D", [64, 128])
def test_fa2_head_shards(dev, world, D):
    # The headline batch B = H = 16 at S = 2048 split over ranks, launched as
    # [1, heads of the rank, S, D] like the bench; the first and last head of
    # the last rank's range against the oracle, plain and causal.
    S = 2048
    sh = shard.shard_heads(16, 16, world, world - 1)
    gd = torch.Generator(device=dev).manual_seed(world * 1000 + D)
    q, k, v = (torch.randn(1, sh.size, S, D, device=dev, generator=gd).half() for _ in range(3))
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    sc = 1 / math.sqrt(D)
    for causal in (False, True):
        o = ops.flash_attention(q, k, v, sc, causal=causal)
        for h in (0, sh.size - 1):
            ref = oracle.attention(qc[0, h], kc[0, h], vc[0, h], sc, causal=causal)
            torch.testing.assert_close(o[0, h].cpu(), ref, **TOL)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fa2_config1_head_shards(dev, world):
    # BASELINE config 1 (B = 1, H = 8, S = 512, D = 64) split over ranks:
    # down to one head a GPU at 8 GPUs.
    sh = shard.shard_heads(1, 8, world, world - 1)
    g = torch.Generator().manual_seed(world)
    q, k, v = (torch.randn(1, sh.size, 512, 64, generator=g).half() for _ in range(3))
    o = ops.flash_attention(q.to(dev), k.to(dev), v.to(dev), 1 / 8)
    for h in range(sh.size):
        torch.testing.assert_close(o[0, h].cpu(), oracle.attention(q[0, h], k[0, h], v[0, h], 1 / 8), **TOL)
