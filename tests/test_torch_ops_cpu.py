"""torch.ops.neso.* registration, checked without a GPU: every operator is
registered, its fake implementation gives the output shape and dtype the
kernel writes (so it traces under FakeTensorMode / torch.compile), and a CPU
input is refused before any library call (there is no CPU kernel)."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import neso_b200.torch_ops as T


def test_every_operator_is_registered():
    for name in T.OPERATORS:
        assert hasattr(torch.ops.neso, name), name


def test_fake_shapes_and_dtypes():
    with FakeTensorMode():
        dev = "cuda"
        x = torch.empty(1000, dtype=torch.float32, device=dev)
        assert torch.ops.neso.vector_add(x, x).shape == (1000,)
        assert torch.ops.neso.scale(x, 0.5).dtype == torch.float32
        q = torch.empty(2, 3, 384, 128, dtype=torch.float16, device=dev)
        table = torch.empty(3, 767, dtype=torch.float32, device=dev)
        o = torch.ops.neso.flash_attention(q, q, q, 0.1, True, table)
        assert o.shape == q.shape and o.dtype == torch.float32
        a = torch.empty(200, 72, dtype=torch.float16, device=dev)
        b = torch.empty(72, 136, dtype=torch.float16, device=dev)
        c = torch.ops.neso.matmul(a, b)
        assert c.shape == (200, 136) and c.dtype == torch.float32
        xq = torch.empty(16, 4096, dtype=torch.float16, device=dev)
        w8 = torch.empty(4096, 11008, dtype=torch.int8, device=dev)
        s8 = torch.empty(11008, dtype=torch.float16, device=dev)
        y = torch.ops.neso.w8a16_matmul(xq, w8, s8)
        assert y.shape == (16, 11008) and y.dtype == torch.float32
        assert torch.ops.neso.w8a16_matmul(xq, w8, None).shape == (16, 11008)
        w4 = torch.empty(2048, 11008, dtype=torch.uint8, device=dev)
        s4 = torch.empty(32, 11008, dtype=torch.float16, device=dev)
        y4 = torch.ops.neso.w4a16_g128_matmul(xq, w4, s4)
        assert y4.shape == (16, 11008) and y4.dtype == torch.float32


def test_cpu_inputs_are_refused():
    x = torch.zeros(8)
    with pytest.raises(ValueError, match="CUDA"):
        torch.ops.neso.vector_add(x, x)
