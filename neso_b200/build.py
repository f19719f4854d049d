"""Build the sm_100a kernel library ``neso_b200/libneso_b200.so`` with nvcc.

Every ``csrc/*.cu`` file is compiled for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` and linked into
one shared library with the static CUDA runtime, so the library loads on a
machine without a GPU driver (the driver is reached lazily through
``cudaGetDriverEntryPoint``). Objects are rebuilt only when a source or header
is newer than them.

Usage: ``python -m neso_b200.build [--force] [-v] [--ptxas-info]``
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libneso_b200.so"
HARNESS_SRC = PKG / "harness" / "neso_harness.cpp"
HARNESS = PKG / "neso_harness"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          f"-I{ROOT / 'include'}", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers()])


def _compile(src: Path, force: bool, ptxas_info: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if not force and not _stale(obj, src):
        return obj, ""
    cmd = [nvcc(), *ARCH, *CFLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return obj, res.stdout + res.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link ``libneso_b200.so``."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        results = list(ex.map(lambda s: _compile(s, force, ptxas_info), sources))
    objs = [o for o, _ in results]
    if verbose or ptxas_info:
        for o, log in results:
            if log:
                print(f"--- {o.name}\n{log}", file=sys.stderr)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    build_harness(force)
    return LIB


def build_harness(force: bool = False) -> Path:
    """Link the native test/bench harness against libneso_b200.so (rpath $ORIGIN)."""
    if (not force and HARNESS.exists() and HARNESS.stat().st_mtime > LIB.stat().st_mtime
            and HARNESS.stat().st_mtime > HARNESS_SRC.stat().st_mtime):
        return HARNESS
    cmd = [nvcc(), *ARCH, "-O2", "-std=c++17", f"-I{ROOT / 'include'}", str(HARNESS_SRC), "-o", str(HARNESS),
           f"-L{PKG}", "-lneso_b200", "-Xlinker", "-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"harness build failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return HARNESS


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/spill report")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))


if __name__ == "__main__":
    main()
