"""Tensor-level API over the C ABI: allocate outputs, derive strides and grids.

These are the calls a PyTorch user makes; each one is a single C-ABI call that
launches the sm_100a kernel on the current CUDA stream. Inputs must already be
CUDA tensors of the stated dtype; nothing is converted or copied implicitly
and there is no CPU path.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from .kernels import current_stream_and_device


def _need(t: torch.Tensor, name: str, dtype: torch.dtype, contiguous: bool = True) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device})")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype} (got {t.dtype})")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def vector_add(x: torch.Tensor, y: torch.Tensor, out: torch.Tensor | None = None,
               block_size: int = 1024) -> torch.Tensor:
    """out = x + y over fp32 vectors (windows/kernels.py:7-15)."""
    _need(x, "x", torch.float32)
    _need(y, "y", torch.float32)
    if x.numel() != y.numel():
        raise ValueError("x and y must have the same number of elements")
    out = torch.empty_like(x) if out is None else out
    _need(out, "out", torch.float32)
    n = x.numel()
    stream = current_stream_and_device([x])
    _lib.call("neso_vector_add", x.data_ptr(), y.data_ptr(), out.data_ptr(), n, block_size,
              (n + block_size - 1) // block_size, 1, 1, stream)
    return out


def scale(x: torch.Tensor, factor: float, out: torch.Tensor | None = None, block_size: int = 1024) -> torch.Tensor:
    """out = x * factor over fp32 vectors (windows/kernels.py:18-22)."""
    _need(x, "x", torch.float32)
    out = torch.empty_like(x) if out is None else out
    _need(out, "out", torch.float32)
    n = x.numel()
    stream = current_stream_and_device([x])
    _lib.call("neso_scale", x.data_ptr(), out.data_ptr(), float(factor), n, block_size,
              (n + block_size - 1) // block_size, 1, 1, stream)
    return out


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
                    causal: bool = False, table: torch.Tensor | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """FA2 forward over contiguous fp16 [B, H, S, D] (D in {64, 128}); fp32 out.

    ``table`` (fp32 [H, 2S-1]) adds table[h, i - j + S - 1] to the logits.
    """
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, n, torch.float16)
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must share one [B, H, S, D] shape")
    B, H, S, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device) if out is None else out
    _need(out, "out", torch.float32)
    stream = current_stream_and_device([q])
    if table is None:
        _lib.call("neso_fa2_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, S, D,
                  float(scale), int(bool(causal)), stream)
    else:
        _need(table, "table", torch.float32)
        if tuple(table.shape) != (H, 2 * S - 1):
            raise ValueError(f"table must be [H, 2S-1] = [{H}, {2 * S - 1}]")
        _lib.call("neso_fa2_fwd_relpos_table", q.data_ptr(), k.data_ptr(), v.data_ptr(), table.data_ptr(),
                  out.data_ptr(), B, H, S, D, float(scale), int(bool(causal)), stream)
    return out


def matmul(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """C (fp32) = A (fp16 [M, K]) @ B (fp16 [K, N]) (tests/test_aot.py:70-99)."""
    _need(a, "a", torch.float16)
    _need(b, "b", torch.float16)
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise ValueError("inner dimensions differ")
    out = torch.empty((M, N), dtype=torch.float32, device=a.device) if out is None else out
    _need(out, "out", torch.float32)
    stream = current_stream_and_device([a])
    _lib.call("neso_matmul_kernel", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, K, 1, N, 1, N, 1,
              128, 128, 32, (M + 127) // 128, (N + 127) // 128, 1, stream)
    return out


def w8a16_matmul(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Y (fp32 [M, N]) = X (fp16 [M, K]) @ (W int8 [K, N] * scale fp16 [N])."""
    _need(x, "x", torch.float16)
    _need(w, "w", torch.int8)
    if scale is not None:
        _need(scale, "scale", torch.float16)
    M, K = x.shape
    N = w.shape[1]
    out = torch.empty((M, N), dtype=torch.float32, device=x.device) if out is None else out
    _need(out, "out", torch.float32)
    stream = current_stream_and_device([x])
    _lib.call("neso_w8a16_matmul_mnk", x.data_ptr(), w.data_ptr(), None if scale is None else scale.data_ptr(),
              out.data_ptr(), M, N, K, stream)
    return out


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """Pack int4 values q [K, N] in [-8, 7] (any integer dtype) into uint8
    [K/2, N]: byte (k/2, n) holds row k even in bits 0-3 and row k odd in bits
    4-7 (two's complement nibbles)."""
    if q.shape[0] % 2:
        raise ValueError("K must be even")
    u = (q.to(torch.int16) & 0xF).to(torch.uint8)
    return (u[0::2] | (u[1::2] << 4)).contiguous()


def w4a16_g128_matmul(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Y (fp32) = sum_g scales[g, n] * sum_{k in g} X[m, k] q[k, n] with packed
    int4 weights wq (uint8 [K/2, N]) and fp16 scales [K/128, N]."""
    _need(x, "x", torch.float16)
    _need(wq, "wq", torch.uint8)
    _need(scales, "scales", torch.float16)
    M, K = x.shape
    N = wq.shape[1]
    out = torch.empty((M, N), dtype=torch.float32, device=x.device) if out is None else out
    _need(out, "out", torch.float32)
    stream = current_stream_and_device([x])
    _lib.call("neso_w4a16_g128_matmul", x.data_ptr(), wq.data_ptr(), scales.data_ptr(), out.data_ptr(), M, N, K,
              stream)
    return out
