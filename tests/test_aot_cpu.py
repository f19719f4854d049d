"""AOT metadata shim and CLI (reference: src/neso/aot_compile.py, src/neso/backend/abi.py,
tests/test_aot.py), CPU only."""
import json

import pytest

from neso_b200 import aot


def test_compile_add_kernel_metadata():
    # tests/test_aot.py:104-138
    r = aot.compile_kernel("add_kernel", "*fp32, *fp32, *fp32, i32, 1024", num_warps=4,
                           grid=["cdiv(n_elements, 1024)", "1", "1"])
    assert r.kernel_name == "add_kernel"
    assert r.constants == {"BLOCK_SIZE": 1024}
    assert r.grid == ["cdiv(n_elements, 1024)", "1", "1"]
    names = [p["name"] for p in r.params]
    assert names == ["x_ptr", "y_ptr", "z_ptr", "n_elements"] and "BLOCK_SIZE" not in names
    meta = json.loads(json.dumps(r.to_metadata()))
    assert set(meta) == {"kernel_name", "params", "constants", "threadgroup_size", "num_warps", "grid"}
    assert meta["constants"]["BLOCK_SIZE"] == 1024
    assert all("rust_type" not in p for p in meta["params"])
    assert meta["threadgroup_size"] == 32 * meta["num_warps"]


def test_compile_matmul_with_hints():
    # tests/test_aot.py:197-202 signature form
    r = aot.compile_kernel("matmul_kernel",
                           "*fp16:16, *fp16:16, *fp32:16, i32, i32, i32, i32, i32, i32, i32, i32, i32, 128, 128, 32",
                           num_warps=8, grid=["cdiv(M,128)", "cdiv(N,128)", "1"])
    assert r.constants == {"BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_K": 32}
    assert [p["index"] for p in r.params] == list(range(12))
    assert r.params[0]["is_pointer"] and not r.params[3]["is_pointer"]


def test_signature_errors_match_reference():
    with pytest.raises(ValueError, match="signature has 3 entries but kernel has 5 arguments"):
        aot.compile_kernel("vector_add", "*fp32, *fp32, *fp32")
    with pytest.raises(ValueError, match="only specialization hints 1 and 16 are supported"):
        aot.compile_kernel("vector_add", "*fp32:8, *fp32, *fp32, i32, 1024")
    with pytest.raises(ValueError, match="must have the form"):
        aot.compile_kernel("vector_add", "*fp32, *fp32, *fp32, i32, 1024", target="neso:2")
    with pytest.raises(ValueError, match="expected a Neso target"):
        aot.compile_kernel("vector_add", "*fp32, *fp32, *fp32, i32, 1024", target="cuda:100:32")
    with pytest.raises(KeyError):
        aot.compile_kernel("square_kernel", "*fp32, *fp32, i32, 1024")
    with pytest.raises(ValueError, match="constexpr"):
        aot.compile_kernel("vector_add", "*fp32, *fp32, *fp32, i32, i32")


def test_parse_signature_reference_semantics():
    ps = aot.parse_signature(["a", "b", "c", "d"], "*fp16:16, i32:1, 64, N", {"N": 7})
    assert ps.constants == {"b": 1, "c": 64, "d": 7}
    assert ps.attributes == {(0,): [["tt.divisibility", 16]]}
    assert ps.triton_signature == {"a": "*fp16", "b": "constexpr", "c": "constexpr", "d": "constexpr"}


def test_cli_writes_metadata(tmp_path):
    out = tmp_path / "vadd"
    rc = aot.main(["--kernel", "vector_add", "--signature", "*fp32, *fp32, *fp32, i32, 256",
                   "--grid", "cdiv(n_elements, 256), 1, 1", "--output", str(out)])
    assert rc == 0
    meta = json.loads((tmp_path / "vadd.json").read_text())
    assert meta["kernel_name"] == "vector_add"
    assert meta["constants"] == {"BLOCK_SIZE": 256}
    assert meta["grid"] == ["cdiv(n_elements, 256)", "1", "1"]
    # argument indices the native harness binds (macos/harness.rs:215-222)
    assert [(p["index"], p["name"]) for p in meta["params"]] == [(0, "x"), (1, "y"), (2, "output"),
                                                                 (3, "n_elements")]
    assert aot.main(["--kernel", "nope", "--signature", "i32"]) == 1


def test_signature_value_forms_and_hints():
    # src/neso/backend/abi.py:59-82: a value body wins over a hint of 1; None
    # is a constexpr; a hint of 1 makes a typed argument the constant 1 while
    # it keeps its written type; a hint of 16 is a divisibility attribute.
    ps = aot.parse_signature(["a", "b", "c"], "64:1, None, *fp32:16")
    assert ps.constants == {"a": 64, "b": None}
    assert ps.source_types == {"a": "constexpr", "b": "constexpr", "c": "*fp32"}
    assert ps.attributes == {(2,): [["tt.divisibility", 16]]}
    ps = aot.parse_signature(["x"], "i32:1")
    assert ps.constants == {"x": 1} and ps.source_types == {"x": "i32"}
    assert ps.triton_signature == {"x": "constexpr"}
    params = aot.build_parameters(["p", "n", "k"], {"p": "*fp16", "k": "constexpr"})
    assert [(q.index, q.name, q.type, q.is_pointer) for q in params] == [(0, "p", "*fp16", True),
                                                                         (1, "n", "i32", False)]


def _elf_symbols(blob: bytes) -> dict[str, int]:
    """Name -> st_info of every symbol in an ELF64 little-endian image."""
    import struct
    shoff = struct.unpack_from("<Q", blob, 0x28)[0]
    shentsize, shnum = struct.unpack_from("<HH", blob, 0x3A)
    secs = [struct.unpack_from("<IIQQQQIIQQ", blob, shoff + i * shentsize) for i in range(shnum)]
    out = {}
    for sec in secs:
        if sec[1] != 2:  # SHT_SYMTAB
            continue
        strtab = secs[sec[6]]
        for off in range(sec[4], sec[4] + sec[5], 24):
            name_off, info = struct.unpack_from("<IB", blob, off)
            end = blob.index(b"\0", strtab[4] + name_off)
            out[blob[strtab[4] + name_off:end].decode()] = info
    return out


needs_nvcc = pytest.mark.skipif(__import__("shutil").which("nvcc") is None
                                and not __import__("os").path.exists("/usr/local/cuda/bin/nvcc"),
                                reason="nvcc not available")


@needs_nvcc
@pytest.mark.parametrize("name,sig", [("vector_add", "*fp32, *fp32, *fp32, i32, 1024"),
                                      ("add_kernel", "*fp32, *fp32, *fp32, i32, 1024"),
                                      ("scale", "*fp32, *fp32, fp32, i32, 256"),
                                      ("softmax_kernel", "*fp32, *fp32, i32, i32, i32, 1024")])
def test_elementwise_kernels_get_a_standalone_cubin(name, sig):
    # The reference writes a compiled library beside the metadata
    # (src/neso/aot_compile.py:56-106); here an sm_100a cubin whose entry has
    # the kernel's name and its runtime parameters in metadata order.
    r = aot.compile_kernel(name, sig, grid=[f"cdiv(n_elements, {sig.split(', ')[-1]})", "1", "1"])
    blob = r.cubin_bytes
    assert blob is not None and blob[:4] == b"\x7fELF"
    assert int.from_bytes(blob[0x12:0x14], "little") == 190  # EM_CUDA
    syms = _elf_symbols(blob)
    assert name in syms and (syms[name] >> 4) == 1 and (syms[name] & 0xF) == 2  # global function
    assert f'extern "C" __global__ void __launch_bounds__({r.threadgroup_size}) {name}(' in r.source
    assert f"{sig.split(', ')[-1]}" in r.source


@needs_nvcc
def test_save_writes_cubin_source_and_metadata(tmp_path):
    r = aot.compile_kernel("vector_add", "*fp32, *fp32, *fp32, i32, 1024", grid=["cdiv(n_elements, 1024)", "1", "1"])
    paths = r.save(str(tmp_path / "vector_add"))
    assert set(paths) == {"cubin", "source", "json"}
    assert (tmp_path / "vector_add.cubin").read_bytes() == r.cubin_bytes
    assert json.loads((tmp_path / "vector_add.json").read_text())["kernel_name"] == "vector_add"


def test_no_cubin_where_there_is_no_standalone_kernel():
    # TMA / tcgen05 kernels are launched through the library's C ABI, and an
    # elementwise signature with other element types has no standalone form.
    r = aot.compile_kernel("matmul_kernel",
                           "*fp16:16, *fp16:16, *fp32:16, i32, i32, i32, i32, i32, i32, i32, i32, i32, 128, 128, 32")
    assert r.cubin_bytes is None and r.source == ""
    r = aot.compile_kernel("add_kernel", "*fp16, *fp16, *fp16, i32, 1024")
    assert r.cubin_bytes is None and r.source == ""
    r = aot.compile_kernel("vector_add", "*fp32, *fp32, *fp32, i32, 1024", emit_cubin=False)
    assert r.cubin_bytes is None and r.save is not None
