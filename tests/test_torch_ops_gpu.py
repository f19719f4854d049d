"""torch.ops.neso.* on the GPU: each operator runs the same kernel as the
tensor API (outputs bit-identical to neso_b200.ops on the same inputs), and
its schema and fake implementation pass torch.library.opcheck."""
import math

import pytest
import torch

import oracle
from neso_b200 import ops
import neso_b200.torch_ops  # noqa: F401

pytestmark = pytest.mark.gpu


def test_operators_match_tensor_api(dev):
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(4099, device=dev, generator=g)
    y = torch.randn(4099, device=dev, generator=g)
    assert torch.equal(torch.ops.neso.vector_add(x, y), ops.vector_add(x, y))
    assert torch.equal(torch.ops.neso.scale(x, -1.75), ops.scale(x, -1.75))

    q, k, v = (torch.randn(2, 3, 300, 64, device=dev, generator=g).half() for _ in range(3))
    table = torch.randn(3, 599, device=dev, generator=g)
    for causal in (False, True):
        for t in (None, table):
            a = torch.ops.neso.flash_attention(q, k, v, 0.125, causal, t)
            assert torch.equal(a, ops.flash_attention(q, k, v, 0.125, causal=causal, table=t))

    A = (torch.randn(200, 72, device=dev, generator=g) / math.sqrt(72)).half()
    B = (torch.randn(72, 136, device=dev, generator=g) / math.sqrt(72)).half()
    assert torch.equal(torch.ops.neso.matmul(A, B), ops.matmul(A, B))

    xq = torch.randn(16, 256, device=dev, generator=g).half()
    w8 = torch.randint(-127, 128, (256, 384), device=dev, dtype=torch.int8, generator=g)
    s8 = (torch.rand(384, device=dev, generator=g) * 0.019 + 0.001).half()
    assert torch.equal(torch.ops.neso.w8a16_matmul(xq, w8, s8), ops.w8a16_matmul(xq, w8, s8))
    assert torch.equal(torch.ops.neso.w8a16_matmul(xq, w8, None), ops.w8a16_matmul(xq, w8))
    q4 = torch.randint(-8, 8, (256, 384), dtype=torch.int8)
    wq = oracle.pack_int4(q4).to(dev)
    s4 = (torch.rand(2, 384, device=dev, generator=g) * 0.019 + 0.001).half()
    assert torch.equal(torch.ops.neso.w4a16_g128_matmul(xq, wq, s4), ops.w4a16_g128_matmul(xq, wq, s4))


def test_opcheck_schema_and_fake(dev):
    g = torch.Generator(device=dev).manual_seed(4)
    q, k, v = (torch.randn(1, 2, 256, 64, device=dev, generator=g).half() for _ in range(3))
    A = torch.randn(128, 64, device=dev, generator=g).half()
    B = torch.randn(64, 128, device=dev, generator=g).half()
    for op, args in ((torch.ops.neso.flash_attention.default, (q, k, v, 0.125, False, None)),
                     (torch.ops.neso.matmul.default, (A, B))):
        torch.library.opcheck(op, args, test_utils=("test_schema", "test_faketensor"))
