"""The library's kernels as PyTorch custom operators, ``torch.ops.neso.*``.

Importing this module registers one operator per tensor-level entry of
``neso_b200.ops``; each calls the same C-ABI entry point on torch's current
stream (CUDA tensors only: there is no CPU kernel, and a CPU input raises as
it does through ``ops``). Every operator also has a fake (meta)
implementation giving the output's shape and dtype without touching a
device, so the operators trace under ``torch.compile``, ``torch.export`` and
FakeTensorMode, where a ctypes call could not run.

    import neso_b200.torch_ops  # noqa: F401  (registers torch.ops.neso.*)
    o = torch.ops.neso.flash_attention(q, k, v, 0.125, False, None)

Outputs are freshly allocated (the ``out=`` buffers of ``ops`` are not part of
the operator schemas, which declare no mutated arguments).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops

_NS = "neso"


@torch.library.custom_op(f"{_NS}::vector_add", mutates_args=())
def vector_add(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """x + y over fp32 vectors (windows/kernels.py:7-15)."""
    return ops.vector_add(x, y)


@vector_add.register_fake
def _vector_add_fake(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    return torch.empty_like(x)


@torch.library.custom_op(f"{_NS}::scale", mutates_args=())
def scale(x: torch.Tensor, factor: float) -> torch.Tensor:
    """x * factor over fp32 vectors (windows/kernels.py:18-22)."""
    return ops.scale(x, factor)


@scale.register_fake
def _scale_fake(x: torch.Tensor, factor: float) -> torch.Tensor:
    return torch.empty_like(x)


@torch.library.custom_op(f"{_NS}::flash_attention", mutates_args=())
def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, softmax_scale: float, causal: bool,
                    table: Optional[torch.Tensor]) -> torch.Tensor:
    """FA2 forward over fp16 [B, H, S, D] (D in {64, 128}), fp32 output; with
    ``table`` (fp32 [H, 2S-1]) the logits add table[h, i - j + S - 1]."""
    return ops.flash_attention(q, k, v, softmax_scale, causal=causal, table=table)


@flash_attention.register_fake
def _flash_attention_fake(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, softmax_scale: float, causal: bool,
                          table: Optional[torch.Tensor]) -> torch.Tensor:
    return q.new_empty(q.shape, dtype=torch.float32)


@torch.library.custom_op(f"{_NS}::matmul", mutates_args=())
def matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp32 C = fp16 A [M, K] @ fp16 B [K, N] (tests/test_aot.py:70-99)."""
    return ops.matmul(a, b)


@matmul.register_fake
def _matmul_fake(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return a.new_empty((a.shape[0], b.shape[1]), dtype=torch.float32)


@torch.library.custom_op(f"{_NS}::w8a16_matmul", mutates_args=())
def w8a16_matmul(x: torch.Tensor, w: torch.Tensor, scale: Optional[torch.Tensor]) -> torch.Tensor:
    """fp32 Y = fp16 X [M, K] @ (int8 W [K, N] * fp16 scale [N]), scale optional
    (tests/test_quantized_matmul.py:67-167, :181-283)."""
    return ops.w8a16_matmul(x, w, scale)


@w8a16_matmul.register_fake
def _w8a16_matmul_fake(x: torch.Tensor, w: torch.Tensor, scale: Optional[torch.Tensor]) -> torch.Tensor:
    return x.new_empty((x.shape[0], w.shape[1]), dtype=torch.float32)


@torch.library.custom_op(f"{_NS}::w4a16_g128_matmul", mutates_args=())
def w4a16_g128_matmul(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 Y = sum_g scales[g, n] * sum_{k in g} X[m, k] q[k, n] over packed
    int4 weights (uint8 [K/2, N]) and fp16 group-128 scales [K/128, N]."""
    return ops.w4a16_g128_matmul(x, wq, scales)


@w4a16_g128_matmul.register_fake
def _w4a16_g128_matmul_fake(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    return x.new_empty((x.shape[0], wq.shape[1]), dtype=torch.float32)


OPERATORS = ("vector_add", "scale", "flash_attention", "matmul", "w8a16_matmul", "w4a16_g128_matmul")
