"""Flash Attention 2 forward on the GPU against the oracle (atol = rtol = 2e-3,
fp32 output) and against the reference's golden vectors at the reference's own
tolerances (tests/test_flash_attention.py:318-341, tests/test_rel_pos_fa2.py:371-373)."""
import math

import numpy as np
import pytest
import torch

import oracle
from neso_b200 import _lib, kernels, ops

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=2e-3)


def _qkv(B, H, S, D, seed=0):
    # BASELINE: Q/K/V ~ N(0, 1) fp16 from a seed
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(B, H, S, D, generator=g).half() for _ in range(3))


def _check(dev, B, H, S, D, causal=False, table=None, seed=0):
    q, k, v = _qkv(B, H, S, D, seed)
    sc = 1.0 / math.sqrt(D)
    o = ops.flash_attention(q.to(dev), k.to(dev), v.to(dev), sc, causal=causal,
                            table=None if table is None else table.to(dev))
    ref = oracle.attention(q, k, v, sc, causal=causal, table=table)
    torch.testing.assert_close(o.cpu(), ref, **TOL)


def test_harness_kat_uniform_softmax(dev):
    # macos/harness.rs:241-271: Q = K = 0 -> O rows = column mean of f16(V); N = 64, d = 64, tol 2e-3
    n, d = 64, 64
    _, _, v = oracle.harness_fa2_values(n, d)
    v16 = v.half()
    z = torch.zeros(n, d, dtype=torch.float16, device=dev)
    o = torch.empty(n, d, device=dev)
    kernels.flash_attention_fwd[(n // 16, 1, 1)](z, z, v16.to(dev), o, n, d, d, 1 / math.sqrt(d))
    exp = v16.float().mean(0, keepdim=True).expand(n, d)
    assert (o.cpu() - exp).abs().max().item() <= 2e-3


@pytest.mark.parametrize("name", ["fa2_N128_d64", "fa2_N256_d128"])
def test_reference_golden_single_head(dev, golden_dir, name):
    g = dict(np.load(golden_dir / f"{name}.npz"))
    N, d = int(g["N"]), int(g["d"])
    q, k, v = (torch.from_numpy(g[t]).half() for t in ("q", "k", "v"))
    o = torch.empty(N, d, device=dev)
    # reference launch: grid (N / BM, 1, 1) with BM = 16 (tests/test_flash_attention.py:290)
    kernels.flash_attention_fwd[(N // 16, 1, 1)](q.to(dev), k.to(dev), v.to(dev), o, N, d, d, float(g["scale"]))
    out = o.cpu().numpy()
    # the reference's f16 criterion on rows 0 and N/2 (tests/test_flash_attention.py:318-341)
    assert np.abs(out[[0, N // 2]] - g["ref_out"][[0, N // 2]]).max() < 0.05
    # BASELINE criterion against the oracle on the same fp16 inputs
    ref = oracle.attention(q, k, v, float(g["scale"]))
    torch.testing.assert_close(o.cpu(), ref, **TOL)


@pytest.mark.parametrize("name", ["relpos_T32_d64_nh2", "relpos_T64_d128_nh4"])
def test_reference_golden_relpos_dense(dev, golden_dir, name):
    g = dict(np.load(golden_dir / f"{name}.npz"))
    T, d, nh = int(g["T"]), int(g["d"]), int(g["nh"])
    qu = torch.from_numpy(g["Q_u"]).half()
    k = torch.from_numpy(g["K"]).half()
    v = torch.from_numpy(g["V"]).half()
    bias = torch.from_numpy(g["rel_bias"]).half()
    o = torch.empty(nh, T, d, dtype=torch.float16, device=dev)
    kernels.rel_pos_fa2_fwd[(T // 16, nh, 1)](qu.to(dev), k.to(dev), v.to(dev), bias.to(dev), o, T, d,
                                              float(g["scale"]), T * d, T * T)
    out = o.float().cpu()
    # the reference's criterion: max abs error < 0.1 vs reference_rel_pos_attention (tests/test_rel_pos_fa2.py:371-373)
    assert np.abs(out.numpy() - g["ref_out"]).max() < 0.1
    ref = oracle.attention(qu, k, v, float(g["scale"]), dense_bias=bias)
    torch.testing.assert_close(out, ref, **TOL)


@pytest.mark.parametrize("T,d,nh", [(2048, 64, 40), (1032, 64, 9), (136, 64, 3), (24, 64, 2),
                                    (1024, 128, 8), (264, 128, 2)])
def test_relpos_dense_sampled_heads(dev, T, d, nh):
    # rel_pos_fa2_fwd at sizes where CTAs walk several query tiles and the
    # last key block and query tile are ragged; heads sampled against the oracle
    g = torch.Generator().manual_seed(T + d + nh)
    q, k, v = (torch.randn(nh, T, d, generator=g).half() for _ in range(3))
    bias = (0.5 * torch.randn(nh, T, T, generator=g)).half()
    o = torch.empty(nh, T, d, dtype=torch.float16, device=dev)
    bm = next(b for b in (128, 64, 32, 16, 8) if T % b == 0)
    sc = 1.0 / math.sqrt(d)
    kernels.rel_pos_fa2_fwd[(T // bm, nh, 1)](q.to(dev), k.to(dev), v.to(dev), bias.to(dev), o, T, d, sc,
                                               T * d, T * T)
    out = o.float().cpu()
    for h in sorted({0, nh // 2, nh - 1}):
        ref = oracle.attention(q[h:h + 1], k[h:h + 1], v[h:h + 1], sc, dense_bias=bias[h:h + 1])
        torch.testing.assert_close(out[h:h + 1], ref, **TOL)


def test_config1_b1_h8_s512_d64(dev):
    _check(dev, 1, 8, 512, 64)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [128, 256, 384, 1000])
@pytest.mark.parametrize("causal", [False, True])
def test_sweep_small(dev, D, S, causal):
    _check(dev, 2, 3, S, D, causal=causal, seed=S + D)


@pytest.mark.parametrize("S", [1, 17, 129])
def test_tiny_and_ragged(dev, S):
    _check(dev, 1, 2, S, 64, seed=S)
    _check(dev, 1, 2, S, 128, causal=True, seed=S)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_relpos_table(dev, D, causal):
    B, H, S = 2, 3, 384
    g = torch.Generator().manual_seed(11)
    table = torch.randn(H, 2 * S - 1, generator=g) * 0.02  # BASELINE: N(0, 0.02)
    _check(dev, B, H, S, D, causal=causal, table=table, seed=12)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S", [1, 77, 300])
def test_relpos_table_ragged_unit_scale(dev, D, causal, S):
    # Ragged S (the last query tile and key block partly past S) and a table of
    # unit scale, so a table entry read at the wrong offset moves the output
    # far past the tolerance; entries past S must be ignored.
    B, H = 2, 3
    g = torch.Generator().manual_seed(S + D)
    table = torch.randn(H, 2 * S - 1, generator=g)
    _check(dev, B, H, S, D, causal=causal, table=table, seed=S)


@pytest.mark.parametrize("D", [64, 128])
def test_relpos_table_many_units_sampled(dev, D):
    # 8 x 16 heads at S = 1000: the D = 128 persistent CTAs each take several
    # work units, so every warp re-stages its table window in its O staging
    # block after the previous unit's stores; causal D = 64 runs two query
    # tiles per CTA. A sample of heads against the oracle.
    B, H, S = 8, 16, 1000
    g = torch.Generator().manual_seed(100 + D)
    q, k, v = (torch.randn(B, H, S, D, generator=g).half() for _ in range(3))
    table = torch.randn(H, 2 * S - 1, generator=g)
    qd, kd, vd, td = q.to(dev), k.to(dev), v.to(dev), table.to(dev)
    for causal in (False, True):
        o = ops.flash_attention(qd, kd, vd, 1 / math.sqrt(D), causal=causal, table=td)
        for (b, h) in [(0, 0), (3, 7), (7, 15)]:
            ref = oracle.attention(q[b, h], k[b, h], v[b, h], 1 / math.sqrt(D), causal=causal,
                                   table=table[h:h + 1])
            torch.testing.assert_close(o[b, h].cpu(), ref, **TOL)


SWEEP_HEADS = [(0, 0), (7, 9), (15, 15)]  # first, a middle and the last (b, h) of B = H = 16


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [128, 256, 512, 1024, 2048])
def test_baseline_sweep_sampled(dev, S, D):
    # BASELINE config 3 at its full shape, B = H = 16: every S and D of the
    # sweep, plain, causal, relative-position table N(0, 0.02) and causal with
    # the table. The unit count (and so the persistent D = 128 scheduler's and
    # the causal pair kernel's work split) changes with S; three heads per
    # point against the oracle.
    B, H = 16, 16
    gd = torch.Generator(device=dev).manual_seed(1000 * D + S)
    q, k, v = (torch.randn(B, H, S, D, device=dev, generator=gd).half() for _ in range(3))
    table = torch.randn(H, 2 * S - 1, device=dev, generator=gd) * 0.02
    qc, kc, vc, tc = q.cpu(), k.cpu(), v.cpu(), table.cpu()
    sc = 1 / math.sqrt(D)
    for causal in (False, True):
        for tab in (None, table):
            o = ops.flash_attention(q, k, v, sc, causal=causal, table=tab)
            for (b, h) in SWEEP_HEADS:
                ref = oracle.attention(qc[b, h], kc[b, h], vc[b, h], sc, causal=causal,
                                       table=None if tab is None else tc[h:h + 1])
                torch.testing.assert_close(o[b, h].cpu(), ref, **TOL)


def _msl_inputs(N, d, seed=42):
    # bench/bench_flash_attention.py:380-384: random.seed(42), then N*d
    # gauss(0, 0.5) draws each for Q, K and V.
    import random
    rnd = random.Random(seed)
    return tuple(torch.tensor([rnd.gauss(0, 0.5) for _ in range(N * d)], dtype=torch.float32).view(N, d)
                 for _ in range(3))


@pytest.mark.parametrize("name", ["flash_attention_fwd_msl", "flash_attention_opt", "flash_attention_d128"])
@pytest.mark.parametrize("use_half", [1, 0])
@pytest.mark.parametrize("N", [256, 2048])
def test_msl_entries(dev, name, use_half, N):
    # The reference's hand-written MSL kernels: one io_type for Q, K, V and O,
    # d_head and scale at run time, grid (N / BM, 1, 1) with BM = 32.
    d = 128 if name == "flash_attention_d128" else 64
    q, k, v = _msl_inputs(N, d)
    dt = torch.float16 if use_half else torch.float32
    qd, kd, vd = (t.to(dt).to(dev) for t in (q, k, v))
    o = torch.zeros(N, d, dtype=dt, device=dev)
    sc = 1.0 / math.sqrt(d)
    getattr(kernels, name)[(N // 32, 1, 1)](qd, kd, vd, o, N, d, sc, BM=32, BN=32)
    out = o.float().cpu()
    ref = oracle.attention(qd.cpu(), kd.cpu(), vd.cpu(), sc)
    # the reference's own check: row 0 within 0.05 (fp16) / 0.01 (fp32)
    assert (out[0] - ref[0]).abs().max().item() < (0.05 if use_half else 0.01)
    torch.testing.assert_close(out, ref, **TOL)


@pytest.mark.parametrize("name", ["fa2_N128_d64", "fa2_N256_d128"])
def test_msl_entry_reference_golden(dev, golden_dir, name):
    # The golden single-head cases through the MSL fp16 entry (O in fp16).
    g = dict(np.load(golden_dir / f"{name}.npz"))
    N, d = int(g["N"]), int(g["d"])
    q, k, v = (torch.from_numpy(g[t]).half() for t in ("q", "k", "v"))
    o = torch.empty(N, d, dtype=torch.float16, device=dev)
    kernels.flash_attention_fwd_msl[(N // 16, 1, 1)](q.to(dev), k.to(dev), v.to(dev), o, N, d, float(g["scale"]),
                                                     BM=16, BN=32)
    out = o.float().cpu()
    assert np.abs(out.numpy()[[0, N // 2]] - g["ref_out"][[0, N // 2]]).max() < 0.05
    torch.testing.assert_close(out, oracle.attention(q, k, v, float(g["scale"])), **TOL)


def test_msl_entry_rejects_mismatched_d_head(dev):
    z = torch.zeros(128, 64, dtype=torch.float16, device=dev)
    with pytest.raises(_lib.NesoError) as ei:
        kernels.flash_attention_fwd_msl[(4, 1, 1)](z, z, z, z, 128, 64, 0.125, d=128)
    assert ei.value.code == _lib.NESO_ERR_INVALID_ARG
    with pytest.raises(_lib.NesoError) as ei:
        kernels.flash_attention_d128[(4, 1, 1)](z, z, z, z, 128, 64, 0.125)
    assert ei.value.code in (_lib.NESO_ERR_UNSUPPORTED, _lib.NESO_ERR_INVALID_ARG)


def test_unsupported_head_dim(dev):
    q = torch.zeros(1, 1, 128, 96, dtype=torch.float16, device=dev)
    with pytest.raises(_lib.NesoError) as ei:
        ops.flash_attention(q, q, q)
    assert ei.value.code == _lib.NESO_ERR_UNSUPPORTED


def test_device_status_clean_after_runs(dev):
    code = torch.zeros(1, dtype=torch.int32)
    rc = _lib.lib().neso_device_status(0, None, None, None, None)
    assert rc == _lib.NESO_OK, _lib.last_error()



def test_dependent_launches_read_the_previous_output(dev):
    # The kernels are launched with programmatic dependent launch: the next
    # kernel's CTAs may start while the previous kernel finishes, and must not
    # read its output before it is complete. A chain of fp16 MSL-entry calls on
    # one stream, each taking the previous output as Q, with no host sync in
    # between; every step is checked against the oracle applied to the
    # previous step's output as the GPU wrote it.
    N, d, steps = 4096, 64, 4
    q, k, v = _msl_inputs(N, d)
    sc = 1.0 / math.sqrt(d)
    kd, vd = k.half().to(dev), v.half().to(dev)
    outs = [q.half().to(dev)] + [torch.empty(N, d, dtype=torch.float16, device=dev) for _ in range(steps)]
    for i in range(steps):
        kernels.flash_attention_fwd_msl[(N // 32, 1, 1)](outs[i], kd, vd, outs[i + 1], N, d, sc, BM=32, BN=32)
    torch.cuda.synchronize(dev)
    kc, vc = kd.cpu(), vd.cpu()
    for i in range(steps):
        ref = oracle.attention(outs[i].cpu(), kc, vc, sc)
        torch.testing.assert_close(outs[i + 1].float().cpu(), ref, **TOL)
