"""Failure detection without a GPU fault: a device wait that nothing satisfies
runs out of its (short) budget, the kernel reports NESO_ERR_DEVICE_TIMEOUT
through the status word and returns, and the context stays usable."""
import ctypes

import pytest
import torch

import oracle
from neso_b200 import _lib, ops

pytestmark = [pytest.mark.gpu, pytest.mark.expects_device_timeout]


def test_bounded_wait_times_out_and_context_survives(dev):
    lib = _lib.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.neso_selftest_wait_timeout(2000, stream)  # 2 ms budget, flag nothing sets
    assert rc == _lib.NESO_ERR_DEVICE_TIMEOUT, _lib.last_error()
    code, where = ctypes.c_int(0), ctypes.c_int(0)
    rc = lib.neso_device_status(0, ctypes.byref(code), ctypes.byref(where), None, None)
    assert rc == _lib.NESO_ERR_DEVICE_TIMEOUT
    assert code.value == 1 and where.value == 0x5E1F
    assert lib.neso_clear_device_status(0) == _lib.NESO_OK
    assert lib.neso_device_status(0, None, None, None, None) == _lib.NESO_OK
    # the context is intact: a normal kernel still runs and is correct
    x = torch.arange(1000, dtype=torch.float32)
    y = ops.vector_add(x.to(dev), x.to(dev))
    assert torch.equal(y.cpu(), oracle.vector_add(x, x))
