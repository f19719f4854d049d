"""The allocation-free W8A16 entry point (neso_w8a16_matmul_mnk_noalloc).

Some callers cannot allocate device memory at the point they run a kernel:
code inside an allocator or memory-pool callback, or a service whose device
memory is fully reserved up front. This entry point takes the same arguments
as neso_w8a16_matmul_mnk but keeps its split-K scratch in a fixed array
compiled into the library. These tests call it through the C ABI, compare it
with the allocating entry point on two calls in a row, check that the calls
leave free device memory unchanged, and that a problem too large for the fixed
scratch is refused with a clear error. The file is named to run last.
"""
import ctypes

import pytest
import torch

from neso_b200 import _lib

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=2e-3)


def _inputs(M, N, K, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).half().to(dev)
    w = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int8).to(dev)
    s = (torch.rand(N, generator=g) * 0.019 + 0.001).half().to(dev)
    return x, w, s


def _call(name, x, w, s, y, M, N, K):
    _lib.call("neso_set_device", x.device.index or 0)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _lib.call(name, x.data_ptr(), w.data_ptr(), s.data_ptr(), y.data_ptr(), M, N, K, stream)


@pytest.mark.parametrize("M", [1, 16])
def test_noalloc_matches_allocating_entry_twice(dev, M):
    N, K = 11008, 4096  # decode-sized W8A16 from BASELINE: split-K, so the scratch is used
    x, w, s = _inputs(M, N, K, 100 + M, dev)
    ref = torch.empty(M, N, device=dev)
    _call("neso_w8a16_matmul_mnk", x, w, s, ref, M, N, K)
    for i in range(2):  # the array keeps the previous call's contents: both calls must be right
        y = torch.full((M, N), float("nan"), device=dev)
        _call("neso_w8a16_matmul_mnk_noalloc", x, w, s, y, M, N, K)
        torch.cuda.synchronize(dev)
        torch.testing.assert_close(y, ref, **TOL)
    assert _lib.lib().neso_device_status(dev.index or 0, None, None, None, None) == _lib.NESO_OK


def test_noalloc_leaves_free_memory_unchanged(dev):
    M, N, K = 4, 11008, 4096
    x, w, s = _inputs(M, N, K, 7, dev)
    y = torch.empty(M, N, device=dev)
    _call("neso_w8a16_matmul_mnk_noalloc", x, w, s, y, M, N, K)  # first call on the device: set-up
    torch.cuda.synchronize(dev)
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(3):
        _call("neso_w8a16_matmul_mnk_noalloc", x, w, s, y, M, N, K)
    torch.cuda.synchronize(dev)
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0


def test_noalloc_rejects_problem_beyond_fixed_scratch(dev):
    # M = 64, N = 2048, K = 65536 splits K nine ways: 9 x 64 x 2048 partial
    # floats > 2^20. Refused on the host before any launch.
    small = torch.zeros(16, device=dev, dtype=torch.float32)
    p = small.data_ptr()
    rc = _lib.lib().neso_w8a16_matmul_mnk_noalloc(p, p, p, p, 64, 2048, 65536,
                                                  torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.NESO_ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()
