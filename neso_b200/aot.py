"""AOT interface of the reference, for the kernels this library implements.

The reference's ``compile_kernel(fn, signature, num_warps, grid, ...)``
(src/neso/aot_compile.py:125-236) compiles a ``@triton.jit`` kernel to Metal and
returns an ``AOTResult`` whose ``to_metadata()`` (aot_compile.py:108-117) native
consumers read. Here the kernels are already compiled for sm_100a inside
``libneso_b200.so``; ``compile_kernel`` resolves the kernel by name, parses the
signature with the reference's grammar (src/neso/backend/abi.py:41-90: bare
literals and known names become constexprs, ``:16`` / ``:1`` are
specialisation hints), checks it against the kernel's argument list, and
returns an ``AOTResult`` with the same metadata schema. ``save(prefix)`` writes
``{prefix}.json`` (the launch metadata; the code is the shared library).

CLI (mirrors ``neso``, aot_compile.py:270-364)::

    python -m neso_b200.aot --kernel vector_add --signature "*fp32, *fp32, *fp32, i32, 1024" \\
        --grid "cdiv(n_elements, 1024), 1, 1" --output vector_add
"""
from __future__ import annotations

import argparse
import json
import sys
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


def _parse_literal(value: str) -> int | float | None:
    try:
        return int(value)
    except ValueError:
        pass
    try:
        return float(value)
    except ValueError:
        return None


def parse_signature(arg_names: Sequence[str], signature: str,
                    namespace: Mapping[str, Any] | None = None) -> ParsedSignature:
    """The reference's signature grammar (src/neso/backend/abi.py:41-90), with
    the same error messages."""
    parts = [part.strip() for part in signature.split(",")]
    if len(parts) != len(arg_names):
        raise ValueError(
            f"signature has {len(parts)} entries but kernel has {len(arg_names)} "
            f"arguments: {list(arg_names)}")
    constants: dict[str, Any] = {}
    hints: dict[tuple[int, ...], int] = {}
    triton_signature: dict[str, str] = {}
    source_types: dict[str, str] = {}
    namespace = namespace or {}
    for index, (name, entry) in enumerate(zip(arg_names, parts)):
        if ":" in entry:
            entry, hint_text = entry.split(":", 1)
            hint = _parse_literal(hint_text)
            if hint not in (1, 16):
                raise ValueError(f"only specialization hints 1 and 16 are supported, got {hint_text!r}")
            hints[(index,)] = int(hint)
            if hint == 1:
                constants[name] = 1
        literal = _parse_literal(entry)
        if literal is not None:
            constants[name] = literal
            source_types[name] = "constexpr"
        elif entry == "None":
            constants[name] = None
            source_types[name] = "constexpr"
        elif entry in namespace:
            constants[name] = namespace[entry]
            source_types[name] = "constexpr"
        else:
            source_types[name] = entry
        triton_signature[name] = "constexpr" if name in constants else entry
    attributes = {path: [["tt.divisibility", 16]] for path, hint in hints.items() if hint == 16}
    return ParsedSignature(triton_signature, constants, attributes, source_types)


def build_parameters(parameter_names: Sequence[str], source_types: Mapping[str, str]) -> list[KernelParameter]:
    """Runtime (non-constexpr) parameters in order, as the reference builds them
    (src/neso/backend/abi.py:93-112)."""
    params = []
    for index, name in enumerate(parameter_names):
        ttype = source_types.get(name, "i32")
        if ttype == "constexpr":
            continue
        params.append(KernelParameter(index=index, name=name, type=ttype,
                                      metal_type=_C_TYPES.get(ttype, ttype), is_pointer=ttype.startswith("*")))
    return params


@dataclass
class AOTResult:
    """Result of ``compile_kernel``; ``to_metadata()`` has the keys of the
    reference's AOTResult.to_metadata() (src/neso/aot_compile.py:108-117)."""

    kernel_name: str
    parameters: list[KernelParameter]
    constants: dict[str, Any]
    threadgroup_size: int
    num_warps: int
    grid: list[str]
    library: str = field(default="")

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
        json_path = prefix.with_suffix(".json")
        json_path.write_text(json.dumps(self.to_metadata(), indent=2))
        return {"json": str(json_path)}


def _resolve(fn) -> _kernels.Kernel:
    name = fn if isinstance(fn, str) else getattr(fn, "__name__", None) or getattr(getattr(fn, "fn", None),
                                                                                    "__name__", None)
    if name not in _kernels.KERNELS:
        raise KeyError(f"kernel {name!r} is not implemented by neso_b200 "
                       f"(available: {', '.join(sorted(_kernels.KERNELS))})")
    return _kernels.KERNELS[name]


def compile_kernel(fn, signature: str, num_warps: int = 4, grid: list[str] | None = None,
                   target: str | None = None, require_metallib: bool = False,
                   emit_metallib: bool = True) -> AOTResult:
    """Resolve ``fn`` (a kernel name, or a function with that ``__name__``) and
    return its launch metadata for ``signature``.

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
    return AOTResult(kernel_name=k.name, parameters=build_parameters(runtime, parsed.source_types),
                     constants=dict(parsed.constants), threadgroup_size=meta["threadgroup_size"],
                     num_warps=meta["num_warps"], grid=grid or ["1", "1", "1"],
                     library=str(Path(__file__).resolve().parent / "libneso_b200.so"))


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
    print(f"  {paths['json']}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
