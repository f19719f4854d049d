"""vector_add / scale on the GPU, bit-exact against the oracle
(windows/kernels.py:7-22; KAT from macos/harness.rs:207-239)."""
import pytest
import torch

import oracle
from neso_b200 import _lib, kernels, ops

pytestmark = pytest.mark.gpu


def _bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    return torch.equal(a.cpu().view(torch.int32), b.cpu().view(torch.int32))


def test_harness_kat_masked_tail(dev):
    x, y = oracle.harness_elementwise_inputs(65537)
    xd, yd = x.to(dev), y.to(dev)
    out = torch.full_like(xd, float("nan"))
    # reference launch shape of the harness: BLOCK 256, grid cdiv(n, 256)
    kernels.vector_add[(65537 + 255) // 256,](xd, yd, out, 65537, BLOCK_SIZE=256)
    assert _bits_equal(out, oracle.vector_add(x, y))
    out2 = torch.full_like(xd, float("nan"))
    kernels.scale[lambda meta: ((meta["n_elements"] + meta["BLOCK_SIZE"] - 1) // meta["BLOCK_SIZE"],)](
        xd, out2, -1.75, 65537, BLOCK_SIZE=256)
    assert _bits_equal(out2, oracle.scale(x, -1.75))


@pytest.mark.parametrize("n", [1, 3, 4, 1023, 1024, 1025, 4097, (1 << 20) + 7])
def test_sizes_bit_exact(dev, n):
    g = torch.Generator().manual_seed(n)
    x = torch.rand(n, generator=g) * 2 - 1
    y = torch.rand(n, generator=g) * 2 - 1
    z = ops.vector_add(x.to(dev), y.to(dev))
    assert _bits_equal(z, oracle.vector_add(x, y))
    s = ops.scale(x.to(dev), 0.5)
    assert _bits_equal(s, oracle.scale(x, 0.5))


def test_misaligned_pointers_take_scalar_path(dev):
    g = torch.Generator().manual_seed(7)
    x = torch.rand(10001, generator=g) * 2 - 1
    y = torch.rand(10001, generator=g) * 2 - 1
    xd, yd = x.to(dev), y.to(dev)
    out = torch.zeros(10001, device=dev)
    # offset every view by one element (4 bytes): not 16-byte aligned
    kernels.vector_add[((10000 + 1023) // 1024,)](xd[1:], yd[1:], out[1:], 10000)
    assert _bits_equal(out[1:], oracle.vector_add(x[1:], y[1:]))
    assert out[0].item() == 0.0


def test_baseline_size_2_28(dev):
    # BASELINE config: n = 2^28, x, y ~ U[-1, 1], a = 0.5
    n = 1 << 28
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.rand(n, device=dev, generator=g) * 2 - 1
    y = torch.rand(n, device=dev, generator=g) * 2 - 1
    z = ops.vector_add(x, y)
    assert _bits_equal(z, oracle.vector_add(x.cpu(), y.cpu()))
    del z
    s = ops.scale(x, 0.5)
    assert _bits_equal(s, oracle.scale(x.cpu(), 0.5))


def test_bad_grid_raises(dev):
    x = torch.zeros(100, device=dev)
    with pytest.raises(_lib.NesoError) as ei:
        kernels.vector_add[(2,)](x, x, x, 100)
    assert ei.value.code == _lib.NESO_ERR_GRID
