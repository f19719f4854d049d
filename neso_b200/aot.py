"""AOT interface of the reference, for the kernels this library implements.

The reference's ``compile_kernel(fn, signature, num_warps, grid, ...)``
(src/neso/aot_compile.py:125-236) compiles a ``@triton.jit`` kernel to Metal and
returns an ``AOTResult`` whose ``to_metadata()`` (aot_compile.py:108-117) native
consumers read. Here the kernels are already compiled for sm_100a inside
``libneso_b200.so``; ``compile_kernel`` resolves the kernel by name, reads the
signature in the reference's grammar (src/neso/backend/abi.py:41-90: numbers,
None and names bound in the kernel's namespace are constexpr values, ``:16``
and ``:1`` are specialisation hints), checks it against the kernel's argument
list, and
returns an ``AOTResult`` with the same metadata schema. ``save(prefix)`` writes
``{prefix}.json`` (the launch metadata). For the elementwise kernels
(``vector_add``, ``add_kernel``, ``scale``) it also writes ``{prefix}.cu`` and
``{prefix}.cubin``: a standalone sm_100a kernel with the reference's parameter
list and Triton program semantics (program ``i`` covers elements
``[i*BLOCK_SIZE, (i+1)*BLOCK_SIZE)``, masked by ``n_elements``), and likewise for
``softmax_kernel`` (program ``i`` = row ``i``), which a native
consumer loads with ``cuModuleLoadData`` and launches from the metadata alone
(grid from ``grid``, block = ``threadgroup_size``, parameters in order), as the
reference's consumers load ``{prefix}.metallib``. The other kernels are TMA /
tcgen05 kernels whose launch needs host-built tensor maps and plans: their
code is ``libneso_b200.so`` and they are launched through its C ABI.

CLI (mirrors ``neso``, aot_compile.py:270-364)::

    python -m neso_b200.aot --kernel vector_add --signature "*fp32, *fp32, *fp32, i32, 1024" \\
        --grid "cdiv(n_elements, 1024), 1, 1" --output vector_add
"""
from __future__ import annotations

import argparse
import json
import subprocess
import sys
import tempfile
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Mapping, Sequence

from . import kernels as _kernels

_C_TYPES = {
    "*fp32": "float*", "*fp16": "__half*", "*bf16": "__nv_bfloat16*", "*i8": "int8_t*", "*u8": "uint8_t*",
    "*i32": "int32_t*", "i32": "int32_t", "i64": "int64_t", "fp32": "float", "fp16": "__half", "u32": "uint32_t",
}


@dataclass(frozen=True)
class ParsedSignature:
    """A parsed signature in the shape the reference's compiler consumes
    (src/neso/backend/abi.py:10-16): per-argument Triton types ("constexpr"
    for specialised arguments), constexpr values, divisibility attributes keyed
    by argument path, and the type each entry was written with."""

    triton_signature: dict[str, str]
    constants: dict[str, Any]
    attributes: dict[tuple[int, ...], list[list[Any]]]
    source_types: dict[str, str]


@dataclass(frozen=True)
class KernelParameter:
    """Same fields as the reference's KernelParameter (src/neso/backend/abi.py:19-27);
    ``metal_type`` carries the C type of the argument."""

    index: int
    name: str
    type: str
    metal_type: str
    is_pointer: bool

    def to_metadata(self) -> dict[str, Any]:
        return asdict(self)


# --- signature grammar -------------------------------------------------------
# One comma-separated entry per kernel argument. An entry is a body with an
# optional ":hint" suffix:
#   body  = <number> | None | <name bound in the kernel's namespace>  -> constexpr value
#         | <Triton type> ("*fp16", "i32", ...)                        -> runtime argument
#   hint  = 16 (pointer / integer divisible by 16: a tt.divisibility attribute)
#         | 1  (the argument is the constant 1)
# Behaviour and error texts follow src/neso/backend/abi.py:41-90.
_HINTS = (1, 16)
_NO_VALUE = object()


def _number(text: str) -> int | float | None:
    """An int if the text is one, else a float if it is one, else None."""
    for conv in (int, float):
        try:
            return conv(text)
        except ValueError:
            continue
    return None


def _value_of(body: str, namespace: Mapping[str, Any]) -> Any:
    """The constexpr value a body denotes, or _NO_VALUE for a type."""
    num = _number(body)
    if num is not None:
        return num
    if body == "None":
        return None
    return namespace[body] if body in namespace else _NO_VALUE


@dataclass(frozen=True)
class SignatureEntry:
    index: int
    name: str
    body: str
    hint: int | None
    value: Any  # _NO_VALUE when the body is a type

    @property
    def written_as_value(self) -> bool:
        return self.value is not _NO_VALUE

    @property
    def constant(self) -> tuple[bool, Any]:
        """(is a constexpr, its value): a value body wins over a hint of 1."""
        if self.written_as_value:
            return True, self.value
        if self.hint == 1:
            return True, 1
        return False, None

    @property
    def source_type(self) -> str:
        return "constexpr" if self.written_as_value else self.body


def _read_entry(index: int, name: str, text: str, namespace: Mapping[str, Any]) -> SignatureEntry:
    body, sep, hint_text = text.partition(":")
    hint = None
    if sep:
        val = _number(hint_text)
        if val not in _HINTS:
            raise ValueError(f"only specialization hints 1 and 16 are supported, got {hint_text!r}")
        hint = int(val)
    body = body.strip()
    return SignatureEntry(index, name, body, hint, _value_of(body, namespace))


def read_signature(arg_names: Sequence[str], signature: str,
                   namespace: Mapping[str, Any] | None = None) -> list[SignatureEntry]:
    """One entry per argument, or ValueError when the counts differ."""
    texts = [t.strip() for t in signature.split(",")]
    if len(texts) != len(arg_names):
        raise ValueError(f"signature has {len(texts)} entries but kernel has {len(arg_names)} "
                         f"arguments: {list(arg_names)}")
    ns = namespace or {}
    return [_read_entry(i, n, t, ns) for i, (n, t) in enumerate(zip(arg_names, texts))]


def parse_signature(arg_names: Sequence[str], signature: str,
                    namespace: Mapping[str, Any] | None = None) -> ParsedSignature:
    """Parse a signature into the structures the reference's compiler takes."""
    entries = read_signature(arg_names, signature, namespace)
    constants = {e.name: e.constant[1] for e in entries if e.constant[0]}
    return ParsedSignature(
        triton_signature={e.name: "constexpr" if e.constant[0] else e.body for e in entries},
        constants=constants,
        attributes={(e.index,): [["tt.divisibility", 16]] for e in entries if e.hint == 16},
        source_types={e.name: e.source_type for e in entries},
    )


def build_parameters(parameter_names: Sequence[str], source_types: Mapping[str, str]) -> list[KernelParameter]:
    """The runtime (non-constexpr) parameters, each at its position among
    `parameter_names`; a name without a written type is an i32 scalar."""
    typed = ((i, n, source_types.get(n, "i32")) for i, n in enumerate(parameter_names))
    return [KernelParameter(i, n, t, _C_TYPES.get(t, t), t.startswith("*")) for i, n, t in typed if t != "constexpr"]


# --- standalone cubins for the elementwise kernels --------------------------
# Each entry: the reference's runtime parameters with the Triton type each must
# have, and the per-element statement. The generated kernel is one CTA per
# program (grid = cdiv(n_elements, BLOCK_SIZE)), its threads striding over the
# program's BLOCK_SIZE elements: the same fp32 operation per element as the
# library kernel, so results are bit-identical to it and to torch.
_STANDALONE = {
    "vector_add": ([("x", "*fp32"), ("y", "*fp32"), ("output", "*fp32"), ("n_elements", "i32")],
                   "output[o] = x[o] + y[o];"),
    "add_kernel": ([("x_ptr", "*fp32"), ("y_ptr", "*fp32"), ("z_ptr", "*fp32"), ("n_elements", "i32")],
                   "z_ptr[o] = x_ptr[o] + y_ptr[o];"),
    "scale": ([("x", "*fp32"), ("output", "*fp32"), ("factor", "fp32"), ("n_elements", "i32")],
              "output[o] = x[o] * factor;"),
}
_OUT_PARAMS = {"output", "z_ptr"}


# softmax_kernel (tests/test_triton_jit.py:55-70): program = row; columns
# [0, min(n_cols, BLOCK_SIZE)); max, sum of exp(x - max), exp(x - max) / sum,
# with the block's threads striding over the row and reducing through shared
# memory.
_SOFTMAX_PARAMS = [("output_ptr", "*fp32"), ("input_ptr", "*fp32"), ("input_row_stride", "i32"),
                   ("output_row_stride", "i32"), ("n_cols", "i32")]


def _softmax_source(block: int, threads: int) -> str:
    w = threads // 32
    return (f"// softmax_kernel: generated by neso_b200.aot for sm_100a. Program blockIdx.x = row;\n"
            f"// columns [0, min(n_cols, {block})); {threads} threads.\n"
            f"__device__ __forceinline__ float warp_max(float v) {{\n"
            f"  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));\n"
            f"  return v;\n}}\n"
            f"__device__ __forceinline__ float warp_sum(float v) {{\n"
            f"  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);\n"
            f"  return v;\n}}\n"
            f"extern \"C\" __global__ void __launch_bounds__({threads}) softmax_kernel(float* __restrict__ output_ptr,\n"
            f"    const float* __restrict__ input_ptr, int input_row_stride, int output_row_stride, int n_cols) {{\n"
            f"  __shared__ float red[{w}];\n"
            f"  const float* row = input_ptr + static_cast<long long>(blockIdx.x) * input_row_stride;\n"
            f"  float* orow = output_ptr + static_cast<long long>(blockIdx.x) * output_row_stride;\n"
            f"  const int nc = n_cols < {block} ? n_cols : {block};\n"
            f"  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;\n"
            f"  float m = __int_as_float(0xff800000);\n"
            f"  for (int c = threadIdx.x; c < nc; c += {threads}) m = fmaxf(m, row[c]);\n"
            f"  m = warp_max(m);\n"
            f"  if (lane == 0) red[warp] = m;\n"
            f"  __syncthreads();\n"
            f"  m = red[0];\n"
            f"  for (int i = 1; i < {w}; ++i) m = fmaxf(m, red[i]);\n"
            f"  __syncthreads();\n"
            f"  float s = 0.f;\n"
            f"  for (int c = threadIdx.x; c < nc; c += {threads}) s += expf(row[c] - m);\n"
            f"  s = warp_sum(s);\n"
            f"  if (lane == 0) red[warp] = s;\n"
            f"  __syncthreads();\n"
            f"  s = red[0];\n"
            f"  for (int i = 1; i < {w}; ++i) s += red[i];\n"
            f"  for (int c = threadIdx.x; c < nc; c += {threads}) orow[c] = __fdiv_rn(expf(row[c] - m), s);\n"
            f"}}\n")


def standalone_source(name: str, source_types: Mapping[str, str], block: int, threads: int) -> str | None:
    """CUDA source of the standalone kernel, or None when `name` has none or
    the signature's types differ from the ones it is written for."""
    if name == "softmax_kernel":
        if block <= 0 or threads <= 0 or threads % 32 or any(source_types.get(p) != t for p, t in _SOFTMAX_PARAMS):
            return None
        return _softmax_source(block, threads)
    spec = _STANDALONE.get(name)
    if spec is None or block <= 0 or threads <= 0:
        return None
    params, stmt = spec
    if any(source_types.get(p) != t for p, t in params):
        return None
    decl = []
    for p, t in params:
        if t == "*fp32":
            decl.append(f"{'' if p in _OUT_PARAMS else 'const '}float* __restrict__ {p}")
        elif t == "fp32":
            decl.append(f"float {p}")
        else:
            decl.append(f"int {p}")
    return (f"// {name}: generated by neso_b200.aot for sm_100a. Program blockIdx.x covers elements\n"
            f"// [blockIdx.x * {block}, (blockIdx.x + 1) * {block}) below n_elements; {threads} threads.\n"
            f"extern \"C\" __global__ void __launch_bounds__({threads}) {name}({', '.join(decl)}) {{\n"
            f"  const long long base = static_cast<long long>(blockIdx.x) * {block};\n"
            f"  for (int i = threadIdx.x; i < {block}; i += {threads}) {{\n"
            f"    const long long o = base + i;\n"
            f"    if (o < n_elements) {stmt}\n"
            f"  }}\n"
            f"}}\n")


def build_cubin(source: str) -> bytes | None:
    """nvcc -cubin for sm_100a; None when nvcc is not available."""
    try:
        from .build import ARCH, nvcc
        compiler = nvcc()
    except (ImportError, RuntimeError):
        return None
    with tempfile.TemporaryDirectory() as d:
        src, out = Path(d) / "k.cu", Path(d) / "k.cubin"
        src.write_text(source)
        res = subprocess.run([compiler, "-cubin", *ARCH, "-O3", "-o", str(out), str(src)],
                             capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc -cubin failed:\n{res.stdout}\n{res.stderr}")
        return out.read_bytes()


@dataclass
class AOTResult:
    """Result of ``compile_kernel``; ``to_metadata()`` has the keys of the
    reference's AOTResult.to_metadata() (src/neso/aot_compile.py:108-117).
    ``source`` / ``cubin_bytes`` hold the standalone kernel where there is one
    (the reference's ``msl_source`` / ``metallib_bytes``), else "" / None."""

    kernel_name: str
    parameters: list[KernelParameter]
    constants: dict[str, Any]
    threadgroup_size: int
    num_warps: int
    grid: list[str]
    library: str = field(default="")
    source: str = field(default="")
    cubin_bytes: bytes | None = field(default=None)

    def to_metadata(self) -> dict[str, Any]:
        return {
            "kernel_name": self.kernel_name,
            "params": [p.to_metadata() for p in self.parameters],
            "constants": self.constants,
            "threadgroup_size": self.threadgroup_size,
            "num_warps": self.num_warps,
            "grid": self.grid,
        }

    @property
    def params(self) -> list[dict[str, Any]]:
        return [p.to_metadata() for p in self.parameters]

    def save(self, output_prefix: str) -> dict[str, str]:
        prefix = Path(output_prefix)
        paths = {}
        if self.cubin_bytes is not None:
            cubin_path = prefix.with_suffix(".cubin")
            cubin_path.write_bytes(self.cubin_bytes)
            paths["cubin"] = str(cubin_path)
        if self.source:
            src_path = prefix.with_suffix(".cu")
            src_path.write_text(self.source)
            paths["source"] = str(src_path)
        json_path = prefix.with_suffix(".json")
        json_path.write_text(json.dumps(self.to_metadata(), indent=2))
        paths["json"] = str(json_path)
        return paths


def _resolve(fn) -> _kernels.Kernel:
    name = fn if isinstance(fn, str) else getattr(fn, "__name__", None) or getattr(getattr(fn, "fn", None),
                                                                                    "__name__", None)
    if name not in _kernels.KERNELS:
        raise KeyError(f"kernel {name!r} is not implemented by neso_b200 "
                       f"(available: {', '.join(sorted(_kernels.KERNELS))})")
    return _kernels.KERNELS[name]


def compile_kernel(fn, signature: str, num_warps: int = 4, grid: list[str] | None = None,
                   target: str | None = None, require_metallib: bool = False,
                   emit_metallib: bool = True, emit_cubin: bool = True) -> AOTResult:
    """Resolve ``fn`` (a kernel name, or a function with that ``__name__``) and
    return its launch metadata for ``signature``; for the elementwise kernels,
    with ``emit_cubin`` and nvcc present, also the standalone sm_100a cubin.

    ``target``, if given, must name this backend ("neso_b200:sm_100a:32");
    ``require_metallib`` cannot be satisfied (there is no Metal toolchain).
    """
    if require_metallib and not emit_metallib:
        raise ValueError("require_metallib=True requires emit_metallib=True")
    if require_metallib:
        raise RuntimeError("no Metal toolchain: the kernels are compiled for sm_100a in libneso_b200.so")
    if target:
        parts = target.split(":")
        if len(parts) != 3:
            raise ValueError("target must have the form 'neso_b200:arch:warp_size'")
        if parts[0] not in ("neso_b200", "neso"):
            raise ValueError(f"expected a Neso target, got {parts[0]!r}")
    k = _resolve(fn)
    arg_names = k.arg_names
    namespace = getattr(getattr(fn, "fn", fn), "__globals__", None) if not isinstance(fn, str) else None
    parsed = parse_signature(arg_names, signature, namespace)
    runtime = [a for a, _ in k.args]
    for name, kind in k.args:
        st = parsed.source_types.get(name)
        if st == "constexpr":
            raise ValueError(f"argument {name!r} is a runtime argument of {k.name} and cannot be a constexpr")
        if (kind == "ptr") != st.startswith("*"):
            raise ValueError(f"argument {name!r} of {k.name} must be {'a pointer' if kind == 'ptr' else 'a scalar'}, "
                             f"signature gives {st!r}")
    for c in k.constexprs:
        if parsed.source_types.get(c) != "constexpr":
            raise ValueError(f"{c!r} is a constexpr of {k.name}; give it a literal value in the signature")
    meta = k.metadata()
    source = ""
    cubin = None
    if emit_cubin:
        block = parsed.constants.get("BLOCK_SIZE")
        src = standalone_source(k.name, parsed.source_types, block if isinstance(block, int) else 0,
                                int(meta["threadgroup_size"]))
        if src is not None:
            cubin = build_cubin(src)
            source = src if cubin is not None else ""
    return AOTResult(kernel_name=k.name, parameters=build_parameters(runtime, parsed.source_types),
                     constants=dict(parsed.constants), threadgroup_size=meta["threadgroup_size"],
                     num_warps=meta["num_warps"], grid=grid or ["1", "1", "1"],
                     library=str(Path(__file__).resolve().parent / "libneso_b200.so"),
                     source=source, cubin_bytes=cubin)


def compile_many(fn, configs: list[dict[str, Any]], target: str | None = None) -> list[AOTResult]:
    return [compile_kernel(fn, cfg["signature"], cfg.get("num_warps", 4), cfg.get("grid"), target) for cfg in configs]


def split_grid(text: str) -> list[str]:
    """Split a grid string on top-level commas only, so "cdiv(n, 256), 1, 1"
    gives three entries (the reference CLI splits on every comma,
    src/neso/aot_compile.py:343, which breaks cdiv(...) expressions)."""
    out, depth, cur = [], 0, []
    for ch in text:
        if ch == "," and depth == 0:
            out.append("".join(cur).strip())
            cur = []
            continue
        depth += ch == "("
        depth -= ch == ")"
        cur.append(ch)
    out.append("".join(cur).strip())
    return out


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="neso_b200 AOT metadata (the reference's `neso` CLI)")
    ap.add_argument("path", nargs="?", help="accepted for compatibility; kernels are resolved by name")
    ap.add_argument("--kernel", "-k", required=True)
    ap.add_argument("--signature", "-s", required=True)
    ap.add_argument("--num-warps", "-w", type=int, default=4)
    ap.add_argument("--grid", "-g", default="1,1,1")
    ap.add_argument("--output", "-o", default=None)
    ap.add_argument("--target", "-t", default=None)
    a = ap.parse_args(argv)
    try:
        res = compile_kernel(a.kernel, a.signature, a.num_warps, split_grid(a.grid), a.target)
    except (KeyError, ValueError, RuntimeError) as e:
        print(f"Error: {e}", file=sys.stderr)
        return 1
    print(f"Kernel: {res.kernel_name}")
    print(f"Threadgroup: {res.threadgroup_size} threads ({res.num_warps} warps)")
    print(f"Constants: {res.constants}")
    for p in res.params:
        print(f"  [{p['index']}] {p['name']}: {p['metal_type']}  ({'buffer' if p['is_pointer'] else 'scalar'})")
    print(f"Grid: ({', '.join(res.grid)})")
    paths = res.save(a.output or a.kernel)
    for key in ("cubin", "source", "json"):
        if key in paths:
            print(f"  {paths[key]}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
