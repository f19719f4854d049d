"""Reference-named kernel handles with Triton-style ``kernel[grid](...)`` launches.

Each handle carries the reference kernel's name, its argument list (runtime
arguments in reference order, then its constexpr parameters) and the C-ABI
entry point that implements it on sm_100a. Launch semantics follow the
reference's Metal launcher (src/neso/backend/driver.py:199-353):

* ``kernel[grid](*args, **constexprs)`` — ``grid`` is a 3-tuple (shorter tuples
  are padded with 1) or a callable taking the dict of launch arguments, as in
  Triton;
* constexpr / specialised arguments are matched by name and never passed as
  kernel buffers (driver.py:205-218, :242-248);
* tensors are passed zero-copy by device pointer (the reference copied every
  tensor through host memory each launch, driver.py:272-283, :335-339);
* scalars are converted to 32-bit int / float (driver.py:284-293);
* a failing launch raises :class:`neso_b200.NesoError` (driver.py:314-317).

Launches are asynchronous on the current torch CUDA stream.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Any, Callable, Sequence

from . import _lib


def _ptr(x: Any, name: str) -> int | None:
    if x is None:
        return None
    if hasattr(x, "data_ptr"):
        if getattr(x, "device", None) is not None and x.device.type != "cuda":
            raise ValueError(f"argument {name!r} must be a CUDA tensor (got device {x.device})")
        return int(x.data_ptr())
    if isinstance(x, int):
        return x
    raise TypeError(f"argument {name!r} must be a tensor or a device pointer, got {type(x).__name__}")


def current_stream_and_device(tensors: Sequence[Any]) -> int:
    """Select the tensors' CUDA device in the library and return the handle of
    torch's current stream on it. The raw-handle query avoids building a
    torch Stream object on every launch (a few microseconds per call)."""
    import torch

    dev = -1
    for t in tensors:
        if getattr(t, "is_cuda", False):
            dev = t.get_device()
            break
    if dev < 0:
        dev = torch.cuda.current_device()
    _lib.call("neso_set_device", dev)
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return int(raw(dev))
    return int(torch.cuda.current_stream(dev).cuda_stream)


@dataclass
class Kernel:
    """A kernel with the reference's name and signature."""

    name: str
    cfunc: str
    args: list[tuple[str, str]]            # (name, kind): kind in {"ptr", "i32", "f32"}
    constexprs: dict[str, Any] = field(default_factory=dict)  # name -> default (None = required)
    infer: dict[str, Callable[[dict], Any]] = field(default_factory=dict)
    # Picks the entry point from the bound arguments when the reference kernel
    # is specialised on an argument's dtype (Triton compiles one per pointer type).
    select: Callable[[dict], str] | None = None

    @property
    def arg_names(self) -> list[str]:
        return [a for a, _ in self.args] + list(self.constexprs)

    def metadata(self) -> dict:
        raw = _lib.lib().neso_kernel_metadata(self.name.encode())
        if raw is None:
            raise KeyError(self.name)
        return json.loads(raw.decode())

    def __getitem__(self, grid) -> Callable[..., None]:
        def launch(*args, **kwargs):
            self.run(grid, *args, **kwargs)
        return launch

    def bind(self, *args, **kwargs) -> dict[str, Any]:
        names = self.arg_names
        if len(args) > len(names):
            raise TypeError(f"{self.name}() takes {len(names)} arguments, got {len(args)}")
        bound: dict[str, Any] = dict(zip(names, args))
        for k, v in kwargs.items():
            if k not in names:
                raise TypeError(f"{self.name}() got an unexpected argument {k!r}")
            if k in bound:
                raise TypeError(f"{self.name}() got multiple values for {k!r}")
            bound[k] = v
        for a, _ in self.args:
            if a not in bound:
                raise TypeError(f"{self.name}() missing argument {a!r}")
        for c, default in self.constexprs.items():
            if c not in bound or bound[c] is None:
                if c in self.infer:
                    bound[c] = self.infer[c](bound)
                elif default is not None:
                    bound[c] = default
                else:
                    raise TypeError(f"{self.name}() missing constexpr {c!r}")
        return bound

    def run(self, grid, *args, **kwargs) -> None:
        bound = self.bind(*args, **kwargs)
        g = grid(bound) if callable(grid) else grid
        g = tuple(int(v) for v in g) + (1,) * (3 - len(tuple(g)))
        if len(g) != 3:
            raise ValueError(f"grid must have at most 3 dimensions, got {g}")
        tensors = [bound[a] for a, kind in self.args if kind == "ptr"]
        stream = current_stream_and_device(tensors)
        cargs: list[Any] = []
        for a, kind in self.args:
            v = bound[a]
            if kind == "ptr":
                cargs.append(_ptr(v, a))
            elif kind == "i32":
                cargs.append(int(v))
            elif kind == "f32":
                cargs.append(float(v))
            else:  # pragma: no cover
                raise AssertionError(kind)
        cargs.extend(int(bound[c]) for c in self.constexprs)
        cargs.extend(g)
        cargs.append(stream)
        _lib.call(self.select(bound) if self.select is not None else self.cfunc, *cargs)


def _last_dim(key: str) -> Callable[[dict], int]:
    return lambda b: int(b[key].shape[-1])


def _is_half(key: str) -> Callable[[dict], int]:
    import torch
    return lambda b: int(b[key].dtype == torch.float16)


def _int32_weights(b: dict) -> str:
    import torch
    w = b["b_int8_ptr"]
    return "neso_w8a16_matmul_kernel_i32" if getattr(w, "dtype", None) == torch.int32 else "neso_w8a16_matmul_kernel"


P, I, F = "ptr", "i32", "f32"

vector_add = Kernel("vector_add", "neso_vector_add",
                    [("x", P), ("y", P), ("output", P), ("n_elements", I)], {"BLOCK_SIZE": 1024})
add_kernel = Kernel("add_kernel", "neso_add_kernel",
                    [("x_ptr", P), ("y_ptr", P), ("z_ptr", P), ("n_elements", I)], {"BLOCK_SIZE": 1024})
scale = Kernel("scale", "neso_scale",
               [("x", P), ("output", P), ("factor", F), ("n_elements", I)], {"BLOCK_SIZE": 1024})
flash_attention_fwd = Kernel(
    "flash_attention_fwd", "neso_flash_attention_fwd",
    [("Q", P), ("K", P), ("V", P), ("O", P), ("N", I), ("stride_qo", I), ("stride_kv", I), ("scale", F)],
    {"d": None}, infer={"d": _last_dim("Q")})
# The hand-written MSL kernels of the reference's benchmarks (bench/bench_flash_attention.py:142-149,
# bench_flash_attention_opt.py:145-152, bench_fa2_d128.py:116-123): one io_type for Q, K, V and O
# (use_half follows Q's dtype unless given), d_head and scale at run time.
_MSL_ARGS = [("Q", P), ("K", P), ("V", P), ("O", P), ("N", I), ("d_head", I), ("scale", F)]
_MSL_CONST = {"BM": 32, "BN": 32, "d": None, "THREADS": 1024, "use_half": None}
_MSL_INFER = {"d": lambda b: int(b["d_head"]), "use_half": _is_half("Q")}
flash_attention_fwd_msl = Kernel("flash_attention_fwd_msl", "neso_flash_attention_fwd_msl", _MSL_ARGS,
                                 dict(_MSL_CONST), dict(_MSL_INFER))
flash_attention_opt = Kernel("flash_attention_opt", "neso_flash_attention_opt", _MSL_ARGS, dict(_MSL_CONST),
                             dict(_MSL_INFER))
flash_attention_d128 = Kernel("flash_attention_d128", "neso_flash_attention_d128", _MSL_ARGS,
                              dict(_MSL_CONST, d=128), dict(_MSL_INFER))
rel_pos_fa2_fwd = Kernel(
    "rel_pos_fa2_fwd", "neso_rel_pos_fa2_fwd",
    [("Q", P), ("K", P), ("V", P), ("bias", P), ("O", P), ("T", I), ("stride", I), ("scale", F),
     ("stride_h", I), ("bias_stride_h", I)],
    {"d": None}, infer={"d": _last_dim("Q")})
matmul_kernel = Kernel(
    "matmul_kernel", "neso_matmul_kernel",
    [("a_ptr", P), ("b_ptr", P), ("c_ptr", P), ("M", I), ("N", I), ("K", I), ("stride_am", I),
     ("stride_ak", I), ("stride_bk", I), ("stride_bn", I), ("stride_cm", I), ("stride_cn", I)],
    {"BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_K": 32})
matmul_tiled = Kernel(
    "matmul_tiled", "neso_matmul_tiled",
    [("a", P), ("b", P), ("c", P), ("K", I), ("stride_am", I), ("stride_bk", I), ("stride_cm", I)],
    {"BM": 128, "BN": 128})
w8a16_matmul = Kernel(
    "w8a16_matmul", "neso_w8a16_matmul",
    [("A", P), ("B", P), ("C", P), ("K", I), ("stride_am", I), ("stride_bk", I), ("stride_cm", I)],
    {"BM": 64, "BN": 64, "BK": 32})
w8a16_scaled_matmul = Kernel(
    "w8a16_scaled_matmul", "neso_w8a16_scaled_matmul",
    [("A", P), ("B", P), ("C", P), ("scale", P), ("K", I), ("stride_am", I), ("stride_bk", I),
     ("stride_cm", I)],
    {"BM": 64, "BN": 64, "BK": 32})
# tests/test_advanced12.py:19-48 (per-tensor fp32 scale; b as int8, or int32 as that test stores it)
w8a16_matmul_kernel = Kernel(
    "w8a16_matmul_kernel", "neso_w8a16_matmul_kernel",
    [("a_ptr", P), ("b_int8_ptr", P), ("c_ptr", P), ("scale_ptr", P), ("M", I), ("N", I), ("K", I),
     ("stride_am", I), ("stride_ak", I), ("stride_bk", I), ("stride_bn", I), ("stride_cm", I), ("stride_cn", I)],
    {"BLOCK_M": None, "BLOCK_N": None, "BLOCK_K": None}, select=_int32_weights)

# LLM building blocks (tests/test_advanced12.py:104-177)
rmsnorm_kernel = Kernel(
    "rmsnorm_kernel", "neso_rmsnorm_kernel",
    [("x_ptr", P), ("weight_ptr", P), ("out_ptr", P), ("row_stride", I), ("n_cols", I), ("eps", F)],
    {"BLOCK_SIZE": None})
residual_rmsnorm_kernel = Kernel(
    "residual_rmsnorm_kernel", "neso_residual_rmsnorm_kernel",
    [("x_ptr", P), ("residual_ptr", P), ("weight_ptr", P), ("out_ptr", P), ("row_stride", I), ("n_cols", I),
     ("eps", F)],
    {"BLOCK_SIZE": None})
rope_kernel = Kernel(
    "rope_kernel", "neso_rope_kernel",
    [("x_ptr", P), ("cos_ptr", P), ("sin_ptr", P), ("out_ptr", P), ("seq_len", I), ("head_dim", I)],
    {"BLOCK_D": None})
silu_kernel = Kernel("silu_kernel", "neso_silu_kernel", [("x_ptr", P), ("out_ptr", P), ("n", I)], {"BLOCK": None})
# tests/test_triton_jit.py:55-70
softmax_kernel = Kernel(
    "softmax_kernel", "neso_softmax_kernel",
    [("output_ptr", P), ("input_ptr", P), ("input_row_stride", I), ("output_row_stride", I), ("n_cols", I)],
    {"BLOCK_SIZE": None})
# tests/test_advanced12.py:54-101 (int8 values held in int32 tensors, as the reference's tests pass them)
per_channel_dequant_kernel = Kernel(
    "per_channel_dequant_kernel", "neso_per_channel_dequant_kernel",
    [("x_int8_ptr", P), ("scale_ptr", P), ("zero_ptr", P), ("out_ptr", P), ("n_rows", I), ("n_cols", I)],
    {"BLOCK_M": None, "BLOCK_N": None})
grouped_dequant_kernel = Kernel(
    "grouped_dequant_kernel", "neso_grouped_dequant_kernel",
    [("x_int8_ptr", P), ("scale_ptr", P), ("zero_ptr", P), ("out_ptr", P), ("n", I), ("group_size", I)],
    {"BLOCK": None})
quantize_kernel = Kernel(
    "quantize_kernel", "neso_quantize_kernel", [("x_ptr", P), ("scale_ptr", P), ("out_ptr", P), ("n", I)],
    {"BLOCK": None})

KERNELS = {k.name: k for k in (vector_add, add_kernel, scale, flash_attention_fwd, flash_attention_fwd_msl,
                                flash_attention_opt, flash_attention_d128, rel_pos_fa2_fwd, matmul_kernel,
                                matmul_tiled, w8a16_matmul, w8a16_scaled_matmul, w8a16_matmul_kernel, rmsnorm_kernel,
                                residual_rmsnorm_kernel, rope_kernel, silu_kernel, softmax_kernel,
                                per_channel_dequant_kernel, grouped_dequant_kernel, quantize_kernel)}
