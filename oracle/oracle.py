"""Torch CPU fp32 restatement of the reference's kernel semantics.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Each function follows a
reference file:line. The reference's own correctness references are pure
Python / NumPy in float64 (tests/test_flash_attention.py:296-339,
tests/test_rel_pos_fa2.py:256-311, tests/test_quantized_matmul.py:288-311);
this oracle states the same mathematics in torch fp32 so it runs at the
benchmark sizes. It is pinned against golden vectors produced by those
reference functions themselves (tests/golden/make_golden.py) and against the
known-answer tests of the reference's native harness (macos/harness.rs).

Parity pins and where they come from:
  * vector_add / scale: bit-exact fp32 (windows/kernels.py:7-22).
  * FA2: softmax((Q K^T) * scale) V in fp32 (tests/test_flash_attention.py:296-312;
    algorithm docstring :1-20). The reference kernel rounds P to the input dtype
    before P.V (:139-142); the oracle does not, so the kernel is compared with a
    tolerance (atol = rtol = 2e-3).
  * rel-pos FA2 (dense bias, reference layout): softmax((Q K^T + bias) * scale) V
    (tests/test_rel_pos_fa2.py:202-206).
  * rel-pos FA2 (table): softmax(Q K^T * scale + table[h, i-j+S-1]) V.
  * GEMM: A.float() @ B.float() (bench/bench_matmul.py:199-201).
  * W8A16: (X @ f16(W)) * scale[n] (tests/test_quantized_matmul.py:288-311).
  * W4A16 g128: sum_g s[g,n] * sum_{k in g} X[m,k] q[k,n], group semantics of
    tests/test_advanced12.py:69-84 (offs // group_size), packing pinned below.
  * RMSNorm / residual RMSNorm, RoPE, SiLU: tests/test_advanced12.py:104-177
    (their own checks :243-298); RoPE is compared bit for bit (plain fp32
    products and sums), the others with a tolerance.
"""
from __future__ import annotations

import math

import numpy as np
import torch

__all__ = [
    "vector_add", "scale", "attention", "attention_rows", "gemm", "w8a16_matmul", "w8a16_matmul_f64",
    "w8a16_matmul_tensor_scale",
    "pack_int4",
    "unpack_int4", "w4a16_g128_matmul", "harness_elementwise_inputs", "harness_fa2_values",
    "rmsnorm", "rope", "silu", "softmax_rows", "per_channel_dequant", "grouped_dequant", "quantize_int8",
]


# ---------------------------------------------------------------- elementwise
def vector_add(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """windows/kernels.py:7-15: output = x + y (fp32)."""
    return (x.float() + y.float())


def scale(x: torch.Tensor, factor: float) -> torch.Tensor:
    """windows/kernels.py:18-22: output = x * factor (fp32; factor as fp32)."""
    return x.float() * torch.tensor(factor, dtype=torch.float32)


def harness_elementwise_inputs(n: int = 65537) -> tuple[torch.Tensor, torch.Tensor]:
    """Known-answer inputs of the native harness (macos/harness.rs:207-209):
    x_i = (i - 1000) * 0.125, y_i = (i mod 97) * -0.25, computed in fp32."""
    i = torch.arange(n, dtype=torch.float32)
    x = (i - 1000.0) * 0.125
    y = torch.remainder(torch.arange(n), 97).to(torch.float32) * -0.25
    return x, y


def harness_fa2_values(n: int, d: int = 64) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """macos/harness.rs:171-183: q_i = ((i%29)-14)*0.01, k_i = ((i%31)-15)*0.01,
    v_i = ((i%17)-8)*0.125 over the flattened [n, d] arrays (fp32)."""
    i = torch.arange(n * d)
    q = (torch.remainder(i, 29).float() - 14.0) * 0.01
    k = (torch.remainder(i, 31).float() - 15.0) * 0.01
    v = (torch.remainder(i, 17).float() - 8.0) * 0.125
    return q.view(n, d), k.view(n, d), v.view(n, d)


# ------------------------------------------------------------ flash attention
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool = False,
              table: torch.Tensor | None = None, dense_bias: torch.Tensor | None = None,
              chunk_heads: int = 16) -> torch.Tensor:
    """Softmax attention over [..., S, D] in fp32 on the CPU.

    * plain: softmax((Q K^T) * scale) V (tests/test_flash_attention.py:296-312).
    * causal: keys j > i masked to -inf.
    * table [H, 2S-1] (fp32): logits + table[h, i - j + S - 1]; the leading
      dims of q are [B, H].
    * dense_bias [..., S, S]: softmax((Q K^T + bias) * scale) V
      (tests/test_rel_pos_fa2.py:202-206).
    Computed chunk-by-chunk over the flattened leading dims so S x S scores fit
    in memory at the benchmark sizes.
    """
    S, D = q.shape[-2], q.shape[-1]
    lead = q.shape[:-2]
    qf = q.reshape(-1, S, D)
    kf = k.reshape(-1, S, D)
    vf = v.reshape(-1, S, D)
    nbh = qf.shape[0]
    out = torch.empty((nbh, S, D), dtype=torch.float32)
    idx = None
    if table is not None:
        H = table.shape[0]
        i = torch.arange(S).view(S, 1)
        j = torch.arange(S).view(1, S)
        idx = (i - j + S - 1)
    mask = None
    if causal:
        mask = torch.ones(S, S, dtype=torch.bool).triu(1)
    bias_f = dense_bias.reshape(-1, S, S) if dense_bias is not None else None
    for c0 in range(0, nbh, chunk_heads):
        c1 = min(nbh, c0 + chunk_heads)
        qs = qf[c0:c1].float()
        ks = kf[c0:c1].float()
        vs = vf[c0:c1].float()
        s = torch.matmul(qs, ks.transpose(-1, -2))
        if bias_f is not None:
            s = (s + bias_f[c0:c1].float()) * scale
        else:
            s = s * scale
        if table is not None:
            heads = torch.arange(c0, c1) % table.shape[0]
            s = s + table.float()[heads][:, idx]
        if mask is not None:
            s = s.masked_fill(mask, float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[c0:c1] = torch.matmul(p, vs)
    return out.reshape(*lead, S, D)


def attention_rows(q: np.ndarray, k: np.ndarray, v: np.ndarray, rows: list[int], scale: float) -> np.ndarray:
    """Row-wise float64 reference for a single head, the way
    tests/test_flash_attention.py:296-339 checks rows 0 and N/2."""
    out = []
    for r in rows:
        s = (k.astype(np.float64) @ q[r].astype(np.float64)) * scale
        e = np.exp(s - s.max())
        w = e / e.sum()
        out.append(w @ v.astype(np.float64))
    return np.stack(out)


# ------------------------------------------------------------------- matmuls
def gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """bench/bench_matmul.py:199-201 / tests/test_aot.py:70-99: C = A @ B, fp32."""
    return torch.matmul(a.float(), b.float())


def w8a16_matmul(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor | None = None) -> torch.Tensor:
    """tests/test_quantized_matmul.py:288-311: C = (X @ f16(W)) [* f32(scale[n])]."""
    c = torch.matmul(x.float(), w.float())
    if scale is not None:
        c = c * scale.float().view(1, -1)
    return c


def w8a16_matmul_f64(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor | None = None) -> torch.Tensor:
    """The same product as w8a16_matmul summed in float64 (the exact value for
    checking fp32 sums whose magnitude makes their rounding order visible)."""
    c = torch.matmul(x.double(), w.double())
    if scale is not None:
        c = c * scale.double().view(1, -1)
    return c


def w8a16_matmul_tensor_scale(a: torch.Tensor, b: torch.Tensor, scale: float) -> torch.Tensor:
    """tests/test_advanced12.py:193: C = A @ (B * scale) in fp32, one scale for
    the whole weight matrix (the kernel, :19-48, multiplies the fp32 sum by it)."""
    return torch.matmul(a.float(), b.float() * float(scale))


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """Pack int4 values q [K, N] (in [-8, 7]) into uint8 [K/2, N]: byte (k/2, n)
    holds row 2i in bits 0-3 and row 2i+1 in bits 4-7, two's complement."""
    assert q.shape[0] % 2 == 0
    u = (q.to(torch.int16) & 0xF).to(torch.uint8)
    return (u[0::2] | (u[1::2] << 4)).contiguous()


def unpack_int4(p: torch.Tensor) -> torch.Tensor:
    """Inverse of pack_int4: uint8 [K/2, N] -> int8 [K, N]."""
    lo = (p & 0xF).to(torch.int16)
    hi = ((p >> 4) & 0xF).to(torch.int16)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    out = torch.empty((p.shape[0] * 2, p.shape[1]), dtype=torch.int8)
    out[0::2] = lo.to(torch.int8)
    out[1::2] = hi.to(torch.int8)
    return out


def w4a16_g128_matmul(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor, group: int = 128) -> torch.Tensor:
    """Y = sum_g s[g, n] * sum_{k in g} X[m, k] q[k, n]; q = unpack_int4(wq).
    Group index g = k // group (tests/test_advanced12.py:69-84)."""
    q = unpack_int4(wq).float()
    s = scales.float().repeat_interleave(group, dim=0)
    return torch.matmul(x.float(), q * s)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
            block: int | None = None) -> torch.Tensor:
    """h / sqrt(sum(h^2) / n_cols + eps) * w, h = x (+ residual), row-wise over
    the first min(block, n_cols) columns, divided by the full n_cols
    (tests/test_advanced12.py:104-120, :135-153; reference check :243-254)."""
    h = x.float() if residual is None else x.float() + residual.float()
    n_cols = h.shape[-1]
    c = n_cols if block is None else min(block, n_cols)
    hc = h[..., :c]
    rms = ((hc * hc).sum(dim=-1, keepdim=True) / n_cols + eps).sqrt()
    return hc / rms * w.float()[:c]  # the columns the kernel writes


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
         block_d: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Rotate pairs (d, d + head_dim/2) of x [seq, head_dim] by cos/sin
    [seq, head_dim/2] (tests/test_advanced12.py:156-176; check :281-298); only
    d < min(block_d, head_dim/2) is rotated and returned."""
    half = x.shape[-1] // 2
    hd = half if block_d is None else min(block_d, half)
    x1, x2 = x[:, :hd].float(), x[:, half:half + hd].float()
    c, s = cos[:, :hd].float(), sin[:, :hd].float()
    return x1 * c - x2 * s, x1 * s + x2 * c  # columns [0, hd) and [half, half + hd)


def silu(x: torch.Tensor) -> torch.Tensor:
    """x * sigmoid(x) (tests/test_advanced12.py:123-132; check :257-265)."""
    xf = x.float()
    return xf * torch.sigmoid(xf)


def softmax_rows(x: torch.Tensor, block: int | None = None) -> torch.Tensor:
    """Row softmax over the first min(block, n_cols) columns
    (tests/test_triton_jit.py:55-70; check :307-325)."""
    c = x.shape[-1] if block is None else min(block, x.shape[-1])
    return torch.softmax(x[..., :c].float(), dim=-1)


def per_channel_dequant(x: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    """(x - zero[col]) * scale[col] (tests/test_advanced12.py:54-67; check :216-226)."""
    return (x.float() - zero.float()[None, :]) * scale.float()[None, :]


def grouped_dequant(x: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, group_size: int) -> torch.Tensor:
    """(x[i] - zero[i // gs]) * scale[i // gs] (tests/test_advanced12.py:69-84; check :229-241)."""
    g = torch.arange(x.numel()) // group_size
    return (x.float() - zero.float()[g]) * scale.float()[g]


def quantize_int8(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """The kernel's rounding (tests/test_advanced12.py:87-101): q = x / scale,
    q + 0.5 or q - 0.5 by sign, truncated toward zero, clamped to [-128, 127]."""
    q = x.float() / scale.float()[0]
    r = torch.where(q >= 0, (q + 0.5).to(torch.int32), (q - 0.5).to(torch.int32))
    return r.clamp(-128, 127).to(torch.int32)


def fa2_flops(B: int, H: int, S: int, D: int, causal: bool = False) -> float:
    """4 * S^2 * D per head (tests/test_flash_attention.py:387); half when causal."""
    f = 4.0 * B * H * S * S * D
    return f / 2 if causal else f


def _selfcheck() -> None:  # pragma: no cover - debugging helper
    x, y = harness_elementwise_inputs(17)
    assert torch.equal(vector_add(x, y), x + y)
    assert math.isclose(float(scale(x, -1.75)[0]), (0 - 1000.0) * 0.125 * -1.75)
