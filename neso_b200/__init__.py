"""neso_b200 — B200-native (sm_100a) implementations of the kernels Neso compiles.

Kernels (hand-written CUDA in ``csrc/``, one shared library ``libneso_b200.so``):
vector_add / scale (128-bit grid-stride HBM streaming), dense fp16 GEMM and
Flash Attention 2 forward (TMA + tcgen05 + TMEM), W8A16 / W4A16 quantized
matmul. ``kernels`` exposes them under the reference kernel names with
Triton-style ``kernel[grid](...)`` launches; ``ops`` is the tensor-level API;
importing ``neso_b200.torch_ops`` registers the same calls as ``torch.ops.neso.*``.
"""
from ._lib import NesoError, NesoLibraryError, lib  # noqa: F401
from . import kernels, ops  # noqa: F401

__all__ = ["NesoError", "NesoLibraryError", "lib", "kernels", "ops"]
