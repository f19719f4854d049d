"""The allocation-free W8A16 entry point (neso_w8a16_matmul_mnk_noalloc).

Some callers cannot allocate device memory at the point they run a kernel:
code inside an allocator or memory-pool callback, or a service whose device
memory is fully reserved up front. This entry point takes the same arguments
as neso_w8a16_matmul_mnk but keeps its split-K scratch in a fixed array
compiled into the library. These tests call it through the C ABI, compare it
with the CPU oracle and with the allocating entry point on two calls in a
row, check that the calls leave free device memory unchanged, and that a
problem whose preferred K split would not fit the fixed scratch runs with
fewer splits and still matches. The file is named to run last.
"""
import pytest
import torch

import oracle
from neso_b200 import _lib

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=2e-3)
SCRATCH_FLOATS = 1 << 20  # the fixed scratch size stated in include/neso_b200.h


def _inputs(M, N, K, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).half()
    w = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int8)
    s = (torch.rand(N, generator=g) * 0.019 + 0.001).half()
    return x.to(dev), w.to(dev), s.to(dev), (x, w, s)


def _call(name, x, w, s, y, M, N, K):
    _lib.call("neso_set_device", x.device.index or 0)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _lib.call(name, x.data_ptr(), w.data_ptr(), s.data_ptr(), y.data_ptr(), M, N, K, stream)


@pytest.mark.parametrize("M", [1, 16])
def test_noalloc_matches_oracle_and_allocating_entry_twice(dev, M):
    N, K = 11008, 4096  # decode-sized W8A16 from BASELINE: split-K, so the scratch is used
    x, w, s, host = _inputs(M, N, K, 100 + M, dev)
    expect = oracle.w8a16_matmul(*host)
    ref = torch.empty(M, N, device=dev)
    _call("neso_w8a16_matmul_mnk", x, w, s, ref, M, N, K)
    for _ in range(2):  # the array keeps the previous call's contents: both calls must be right
        y = torch.full((M, N), float("nan"), device=dev)
        _call("neso_w8a16_matmul_mnk_noalloc", x, w, s, y, M, N, K)
        torch.cuda.synchronize(dev)
        torch.testing.assert_close(y, ref, **TOL)
        torch.testing.assert_close(y.cpu(), expect, **TOL)
    assert _lib.lib().neso_device_status(dev.index or 0, None, None, None, None) == _lib.NESO_OK


def test_noalloc_leaves_free_memory_unchanged(dev):
    M, N, K = 4, 11008, 4096
    x, w, s, _ = _inputs(M, N, K, 7, dev)
    y = torch.empty(M, N, device=dev)
    _call("neso_w8a16_matmul_mnk_noalloc", x, w, s, y, M, N, K)  # first call on the device: set-up
    torch.cuda.synchronize(dev)
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(3):
        _call("neso_w8a16_matmul_mnk_noalloc", x, w, s, y, M, N, K)
    torch.cuda.synchronize(dev)
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0


def test_noalloc_large_problem_splits_within_fixed_scratch(dev):
    # M = 64, N = 2048, K = 16384 with full-size buffers: on a 148-SM B200
    # the allocating entry point splits K nine ways, 9 x 64 x 2048 partial
    # floats, more than the fixed scratch holds; the allocation-free entry
    # point splits K only as far as the partial sums fit and must still give
    # the same result. The reference sum is taken in float64: two fp32 sums of
    # 16k terms in different orders differ by about 1e-3 at these magnitudes.
    M, N, K = 64, 2048, 16384
    assert 9 * M * N > SCRATCH_FLOATS
    x, w, s, (xh, wh, sh) = _inputs(M, N, K, 11, dev)
    expect = (xh.double() @ wh.double() * sh.double().view(1, -1)).float()
    for _ in range(2):
        y = torch.full((M, N), float("nan"), device=dev)
        _call("neso_w8a16_matmul_mnk_noalloc", x, w, s, y, M, N, K)
        torch.cuda.synchronize(dev)
        torch.testing.assert_close(y.cpu(), expect, **TOL)


def test_noalloc_empty_k_writes_zeros(dev):
    M, N = 3, 64
    x = torch.empty(M, 0, device=dev, dtype=torch.float16)
    w = torch.empty(0, N, device=dev, dtype=torch.int8)
    s = torch.ones(N, device=dev, dtype=torch.float16)
    y = torch.full((M, N), float("nan"), device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = _lib.lib().neso_w8a16_matmul_mnk_noalloc(x.data_ptr() or None, w.data_ptr() or None, s.data_ptr(),
                                                  y.data_ptr(), M, N, 0, stream)
    assert rc == _lib.NESO_OK, _lib.last_error()
    torch.cuda.synchronize(dev)
    assert torch.equal(y.cpu(), torch.zeros(M, N))
