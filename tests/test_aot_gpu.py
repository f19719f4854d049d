"""The AOT output used the way a native consumer uses it: load the .cubin with
the CUDA driver, look the kernel up by the metadata's kernel_name, launch it
with the metadata's grid and threadgroup size and the parameters in metadata
order, and compare with the oracle: bit for bit for the elementwise kernels
(windows/kernels.py:7-22, tests/test_aot.py:17-28), at the row-kernel tests'
tolerance for softmax_kernel (tests/test_triton_jit.py:55-70)."""
import ctypes
import math

import pytest
import torch

import oracle
from neso_b200 import aot

pytestmark = pytest.mark.gpu


def _driver():
    cu = ctypes.CDLL("libcuda.so.1")
    cu.cuModuleLoadData.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
    cu.cuModuleGetFunction.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_char_p]
    cu.cuModuleUnload.argtypes = [ctypes.c_void_p]
    cu.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 7 + [ctypes.c_void_p,
                                                                             ctypes.POINTER(ctypes.c_void_p),
                                                                             ctypes.c_void_p]
    return cu


def _launch(result, grid, args):
    """Launch the AOT kernel on `grid` CTAs of threadgroup_size threads."""
    cu = _driver()
    mod, fn = ctypes.c_void_p(), ctypes.c_void_p()
    assert cu.cuModuleLoadData(ctypes.byref(mod), result.cubin_bytes) == 0
    try:
        assert cu.cuModuleGetFunction(ctypes.byref(fn), mod, result.kernel_name.encode()) == 0
        holders = []
        for meta, a in zip(result.params, args):
            if meta["is_pointer"]:
                holders.append(ctypes.c_uint64(a.data_ptr()))
            elif meta["type"] == "fp32":
                holders.append(ctypes.c_float(a))
            else:
                holders.append(ctypes.c_int32(a))
        kp = (ctypes.c_void_p * len(holders))(*[ctypes.addressof(h) for h in holders])
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        assert cu.cuLaunchKernel(fn, grid, 1, 1, result.threadgroup_size, 1, 1, 0, stream, kp, None) == 0
        torch.cuda.synchronize()
    finally:
        cu.cuModuleUnload(mod)


@pytest.mark.parametrize("name", ["vector_add", "add_kernel"])
@pytest.mark.parametrize("n", [65537, (1 << 20) + 3])
def test_aot_cubin_add(dev, name, n):
    r = aot.compile_kernel(name, "*fp32, *fp32, *fp32, i32, 1024", grid=["cdiv(n_elements, 1024)", "1", "1"])
    if r.cubin_bytes is None:
        pytest.skip("nvcc not available")
    g = torch.Generator().manual_seed(n)
    x = torch.rand(n, generator=g) * 2 - 1
    y = torch.rand(n, generator=g) * 2 - 1
    xd, yd = x.to(dev), y.to(dev)
    z = torch.full((n + 5,), 7.0, device=dev)
    _launch(r, math.ceil(n / 1024), [xd, yd, z, n])
    assert torch.equal(z[:n].cpu(), oracle.vector_add(x, y))
    assert torch.all(z[n:] == 7.0)  # nothing written past n_elements


def test_aot_cubin_scale(dev):
    n = 100003
    r = aot.compile_kernel("scale", "*fp32, *fp32, fp32, i32, 256", grid=["cdiv(n_elements, 256)", "1", "1"])
    if r.cubin_bytes is None:
        pytest.skip("nvcc not available")
    x = torch.rand(n, generator=torch.Generator().manual_seed(3)) * 2 - 1
    out = torch.empty(n, device=dev)
    _launch(r, math.ceil(n / 256), [x.to(dev), out, -1.75, n])
    assert torch.equal(out.cpu(), oracle.scale(x, -1.75))


@pytest.mark.parametrize("M,N,block", [(37, 1000, 1024), (5, 3000, 2048), (8, 700, 512)])
def test_aot_cubin_softmax(dev, M, N, block):
    # tests/test_triton_jit.py:55-70 signature, grid = rows; with BLOCK_SIZE <
    # n_cols only the first BLOCK_SIZE columns are written.
    r = aot.compile_kernel("softmax_kernel", f"*fp32, *fp32, i32, i32, i32, {block}", grid=["n_rows", "1", "1"])
    if r.cubin_bytes is None:
        pytest.skip("nvcc not available")
    x = torch.randn(M, N, generator=torch.Generator().manual_seed(M * N)) * 4
    out = torch.full((M, N + 3), 7.0, device=dev)
    _launch(r, M, [out, x.to(dev), N, N + 3, N])
    c = min(block, N)
    torch.testing.assert_close(out[:, :c].cpu(), oracle.softmax_rows(x, block), atol=1e-6, rtol=1e-5)
    assert torch.all(out[:, c:] == 7.0)
