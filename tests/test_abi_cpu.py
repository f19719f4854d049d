"""C-ABI checks that need no GPU: the library loads, exports exactly what the
header declares, reports reference-schema metadata, and rejects invalid
launches (wrong reference grid, unsupported strides, bad constexprs) before
touching the device."""
import ctypes
import json

import pytest

from neso_b200 import _lib


def test_library_loads_and_exports_every_header_symbol():
    lib = _lib.lib()
    declared = _lib.header_functions()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/neso_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(declared)
    assert lib.neso_version() >= 100


def test_metadata_matches_reference_schema():
    lib = _lib.lib()
    # keys of AOTResult.to_metadata() (src/neso/aot_compile.py:108-117)
    keys = {"kernel_name", "params", "constants", "threadgroup_size", "num_warps", "grid"}
    for name in ["vector_add", "add_kernel", "scale", "flash_attention_fwd", "rel_pos_fa2_fwd", "matmul_kernel",
                 "matmul_tiled", "w8a16_matmul", "w8a16_scaled_matmul", "fa2_fwd", "fa2_fwd_relpos_table",
                 "w8a16_matmul_mnk", "w4a16_g128_matmul", "flash_attention_fwd_msl", "flash_attention_opt",
                 "flash_attention_d128", "w8a16_matmul_kernel"]:
        meta = json.loads(lib.neso_kernel_metadata(name.encode()).decode())
        assert set(meta) == keys, name
        assert meta["kernel_name"] == name
        assert meta["threadgroup_size"] == 32 * meta["num_warps"]
        assert len(meta["grid"]) == 3
        for i, p in enumerate(meta["params"]):
            # KernelParameter fields (src/neso/backend/abi.py:19-27) and no rust_type (tests/test_aot.py:136)
            assert {"index", "name", "type", "metal_type", "is_pointer"} <= set(p)
            assert "rust_type" not in p
            assert p["index"] == i
            assert p["is_pointer"] == p["type"].startswith("*")
    assert lib.neso_kernel_metadata(b"no_such_kernel") is None
    add = json.loads(lib.neso_kernel_metadata(b"add_kernel").decode())
    assert add["constants"] == {"BLOCK_SIZE": 1024}
    assert [p["name"] for p in add["params"]] == ["x_ptr", "y_ptr", "z_ptr", "n_elements"]


def test_scale_metadata_argument_indices_match_harness():
    # macos/harness.rs:229-236 binds factor at index 2 and n at index 3.
    meta = json.loads(_lib.lib().neso_kernel_metadata(b"scale").decode())
    idx = {p["name"]: p["index"] for p in meta["params"]}
    assert idx["factor"] == 2 and idx["n_elements"] == 3


@pytest.mark.parametrize("n,block,grid,expect", [
    (10, 1024, (2, 1, 1), _lib.NESO_ERR_GRID),
    (65537, 256, (256, 1, 1), _lib.NESO_ERR_GRID),
    (65537, 256, (257, 2, 1), _lib.NESO_ERR_GRID),
    (10, 1000, (1, 1, 1), _lib.NESO_ERR_INVALID_ARG),   # BLOCK_SIZE not a power of two
    (-1, 1024, (0, 1, 1), _lib.NESO_ERR_INVALID_ARG),
])
def test_elementwise_rejects_bad_launch(n, block, grid, expect):
    lib = _lib.lib()
    assert lib.neso_vector_add(None, None, None, n, block, *grid, None) == expect
    assert _lib.last_error()
    assert lib.neso_scale(None, None, 1.0, n, block, *grid, None) == expect


def test_zero_elements_is_a_no_op():
    assert _lib.lib().neso_vector_add(None, None, None, 0, 1024, 0, 1, 1, None) == _lib.NESO_OK


@pytest.mark.parametrize("N,grid", [(128, (3, 1, 1)), (128, (256, 1, 1)), (128, (128, 1, 1)), (128, (8, 2, 1))])
def test_fa2_reference_grid_checked(N, grid):
    # grid (N/BM, 1, 1) with BM a power of two in [8, 128] (tests/test_flash_attention.py:290)
    rc = _lib.lib().neso_flash_attention_fwd(None, None, None, None, N, 64, 64, 0.125, 64, *grid, None)
    assert rc == _lib.NESO_ERR_GRID


def test_matmul_grid_and_strides_checked():
    lib = _lib.lib()
    rc = lib.neso_matmul_kernel(None, None, None, 256, 256, 64, 64, 1, 256, 1, 256, 1, 128, 128, 32, 3, 2, 1, None)
    assert rc == _lib.NESO_ERR_GRID
    rc = lib.neso_matmul_kernel(None, None, None, 256, 256, 64, 64, 2, 256, 1, 256, 1, 128, 128, 32, 2, 2, 1, None)
    assert rc == _lib.NESO_ERR_UNSUPPORTED
    rc = lib.neso_matmul_kernel(None, None, None, 256, 256, 64, 64, 1, 256, 1, 256, 1, 0, 128, 32, 2, 2, 1, None)
    assert rc == _lib.NESO_ERR_INVALID_ARG


@pytest.mark.parametrize("fn", ["neso_flash_attention_fwd_msl", "neso_flash_attention_opt", "neso_flash_attention_d128"])
def test_msl_fa2_entries_check_launch_before_the_device(fn):
    # bench/bench_flash_attention.py:375: grid (N // BM, 1, 1); d_head equal to the compiled d.
    f = getattr(_lib.lib(), fn)
    d = 128
    # (Q, K, V, O, N, d_head, scale, BM, BN, d, THREADS, use_half, grid, stream)
    assert f(None, None, None, None, 256, d, 0.1, 32, 32, d, 1024, 1, 7, 1, 1, None) == _lib.NESO_ERR_GRID
    assert f(None, None, None, None, 250, d, 0.1, 32, 32, d, 1024, 1, 7, 1, 1, None) == _lib.NESO_ERR_GRID
    assert f(None, None, None, None, 256, 64, 0.1, 32, 32, d, 1024, 1, 8, 1, 1, None) == _lib.NESO_ERR_INVALID_ARG
    assert f(None, None, None, None, 256, d, 0.1, 32, 32, d, 1024, 2, 8, 1, 1, None) == _lib.NESO_ERR_INVALID_ARG
    assert f(None, None, None, None, 256, 96, 0.1, 32, 32, 96, 1024, 1, 8, 1, 1, None) == _lib.NESO_ERR_UNSUPPORTED
    assert f(None, None, None, None, 256, d, 0.1, 32, 32, d, 1024, 1, 8, 1, 1, None) == _lib.NESO_ERR_INVALID_ARG  # null


def test_flash_attention_d128_rejects_d64():
    rc = _lib.lib().neso_flash_attention_d128(None, None, None, None, 256, 64, 0.1, 32, 32, 64, 1024, 1, 8, 1, 1, None)
    assert rc == _lib.NESO_ERR_UNSUPPORTED


@pytest.mark.parametrize("fn", ["neso_w8a16_matmul_kernel", "neso_w8a16_matmul_kernel_i32"])
def test_w8a16_tensor_scale_checks_launch_before_the_device(fn):
    # tests/test_advanced12.py:188-196: grid (cdiv(M, BLOCK_M), cdiv(N, BLOCK_N)).
    f = getattr(_lib.lib(), fn)
    ok_args = (32, 32, 32, 32, 1, 32, 1, 32, 1, 32, 32, 32)
    assert f(None, None, None, None, *ok_args, 2, 1, 1, None) == _lib.NESO_ERR_GRID
    bad_stride = (32, 32, 32, 32, 2, 32, 1, 32, 1, 32, 32, 32)
    assert f(None, None, None, None, *bad_stride, 1, 1, 1, None) == _lib.NESO_ERR_UNSUPPORTED
    assert f(None, None, None, None, *ok_args, 1, 1, 1, None) == _lib.NESO_ERR_INVALID_ARG  # null scale
    zero_block = (32, 32, 32, 32, 1, 32, 1, 32, 1, 0, 32, 32)
    assert f(None, None, None, None, *zero_block, 1, 1, 1, None) == _lib.NESO_ERR_INVALID_ARG


def test_error_string_is_thread_local():
    import threading

    lib = _lib.lib()
    lib.neso_vector_add(None, None, None, 10, 1024, 7, 1, 1, None)
    main_msg = _lib.last_error()
    seen = {}

    def worker():
        seen["msg"] = _lib.last_error()

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert "grid" in main_msg
    assert seen["msg"] == ""


def test_status_codes_match_header():
    text = _lib.HEADER_PATH.read_text()
    for name in ["NESO_OK", "NESO_ERR_INVALID_ARG", "NESO_ERR_MISALIGNED", "NESO_ERR_UNSUPPORTED", "NESO_ERR_GRID",
                 "NESO_ERR_LAUNCH", "NESO_ERR_DEVICE_TIMEOUT", "NESO_ERR_NO_DEVICE"]:
        val = getattr(_lib, name)
        assert f"#define {name} ({val})" in text or f"#define {name} {val}" in text


class _FakeCudaTensor:
    def __init__(self, index):
        self.is_cuda = True
        self._index = index

    def get_device(self):
        return self._index


class _FakeCpuTensor:
    is_cuda = False

    def get_device(self):
        return -1


def test_launch_stream_and_device_selection(monkeypatch):
    # Host logic of every launch: the first CUDA tensor picks the device, the
    # library is switched to it, and torch's current stream on that device is
    # passed as a raw handle (falling back to the Stream object without the
    # raw query).
    import torch

    from neso_b200 import kernels

    calls = []
    monkeypatch.setattr(_lib, "call", lambda name, *args: calls.append((name, args)))
    monkeypatch.setattr(torch._C, "_cuda_getCurrentRawStream", lambda dev: 0x1000 + dev, raising=False)
    assert kernels.current_stream_and_device([3, _FakeCpuTensor(), _FakeCudaTensor(2), _FakeCudaTensor(5)]) == 0x1002
    assert calls == [("neso_set_device", (2,))]

    calls.clear()
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 1)
    assert kernels.current_stream_and_device([_FakeCpuTensor()]) == 0x1001
    assert calls == [("neso_set_device", (1,))]

    class _Stream:
        cuda_stream = 0xBEEF

    monkeypatch.delattr(torch._C, "_cuda_getCurrentRawStream")
    monkeypatch.setattr(torch.cuda, "current_stream", lambda dev: _Stream())
    assert kernels.current_stream_and_device([_FakeCudaTensor(0)]) == 0xBEEF


def test_rowops_reject_bad_launch_before_the_device():
    lib = _lib.lib()
    G, I = _lib.NESO_ERR_GRID, _lib.NESO_ERR_INVALID_ARG
    assert lib.neso_rmsnorm_kernel(None, None, None, 128, 128, 1e-5, 100, 32, 1, 1, None) == I  # BLOCK not 2^k
    assert lib.neso_rmsnorm_kernel(None, None, None, 128, 128, 1e-5, 128, 32, 2, 1, None) == G
    assert lib.neso_residual_rmsnorm_kernel(None, None, None, None, 128, 128, 1e-5, 128, 32, 1, 3, None) == G
    assert lib.neso_rope_kernel(None, None, None, None, 16, 64, 32, 15, 1, 1, None) == G   # grid != seq_len
    assert lib.neso_rope_kernel(None, None, None, None, 16, 64, 24, 16, 1, 1, None) == I   # BLOCK_D not 2^k
    assert lib.neso_silu_kernel(None, None, 2048, 256, 9, 1, 1, None) == G                 # cdiv(2048, 256) = 8
    assert lib.neso_silu_kernel(None, None, 2048, 300, 7, 1, 1, None) == I
    # empty problems are no-ops
    assert lib.neso_rmsnorm_kernel(None, None, None, 128, 128, 1e-5, 128, 0, 1, 1, None) == _lib.NESO_OK
    assert lib.neso_rope_kernel(None, None, None, None, 0, 64, 32, 0, 1, 1, None) == _lib.NESO_OK
    assert lib.neso_silu_kernel(None, None, 0, 256, 0, 1, 1, None) == _lib.NESO_OK
    assert lib.neso_softmax_kernel(None, None, 128, 128, 128, 96, 16, 1, 1, None) == I              # BLOCK not 2^k
    assert lib.neso_per_channel_dequant_kernel(None, None, None, None, 32, 64, 32, 32, 1, 1, 1, None) == G  # want (1, 2, 1)
    assert lib.neso_grouped_dequant_kernel(None, None, None, None, 1024, 0, 256, 4, 1, 1, None) == I  # group 0
    assert lib.neso_quantize_kernel(None, None, None, 1024, 256, 5, 1, 1, None) == G
    for name in ("rmsnorm_kernel", "residual_rmsnorm_kernel", "rope_kernel", "silu_kernel", "softmax_kernel",
                 "per_channel_dequant_kernel", "grouped_dequant_kernel", "quantize_kernel"):
        meta = json.loads(lib.neso_kernel_metadata(name.encode()).decode())
        assert meta["kernel_name"] == name


def test_row_kernel_handles_bind_like_the_reference_launcher():
    # Reference launches (tests/test_advanced12.py:249, :275, :295; tests/test_triton_jit.py:311):
    # runtime arguments in order, BLOCK constexprs by name and required (no default is invented).
    from neso_b200 import kernels

    b = kernels.rmsnorm_kernel.bind("x", "w", "out", 128, 128, 1e-5, BLOCK_SIZE=128)
    assert list(b) == ["x_ptr", "weight_ptr", "out_ptr", "row_stride", "n_cols", "eps", "BLOCK_SIZE"]
    b = kernels.softmax_kernel.bind("out", "x", 128, 128, 128, BLOCK_SIZE=256)
    assert b["output_ptr"] == "out" and b["input_ptr"] == "x" and b["BLOCK_SIZE"] == 256
    b = kernels.per_channel_dequant_kernel.bind("x", "s", "z", "o", 32, 64, BLOCK_M=32, BLOCK_N=32)
    assert (b["n_rows"], b["n_cols"], b["BLOCK_M"], b["BLOCK_N"]) == (32, 64, 32, 32)
    for k, args in ((kernels.rope_kernel, ("x", "c", "s", "o", 16, 64)), (kernels.silu_kernel, ("x", "o", 2048)),
                    (kernels.quantize_kernel, ("x", "s", "o", 1024)),
                    (kernels.grouped_dequant_kernel, ("x", "s", "z", "o", 1024, 128))):
        with pytest.raises(TypeError, match="constexpr"):
            k.bind(*args)
    assert set(kernels.KERNELS) >= {"rmsnorm_kernel", "residual_rmsnorm_kernel", "rope_kernel", "silu_kernel",
                                    "softmax_kernel", "per_channel_dequant_kernel", "grouped_dequant_kernel",
                                    "quantize_kernel"}
