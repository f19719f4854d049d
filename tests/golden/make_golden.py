"""Generate the golden vectors in tests/golden/*.npz from the reference itself.

The reference's correctness references are plain Python / NumPy functions in
its test scripts (tests/test_rel_pos_fa2.py:256-311 and
tests/test_quantized_matmul.py:288-311). Those scripts import PyObjC's
``Metal`` at module level and create a device, so this generator installs a
stand-in ``Metal`` module (no GPU work is ever dispatched through it) and then
calls the reference functions on the reference's own seeded inputs.

This script needs a checkout of the reference, named by the NESO_REFERENCE
environment variable or the first command-line argument; the GPU box never
runs it. The generated ``.npz`` files are committed and read by
tests/test_oracle_golden.py.

Run: NESO_REFERENCE=<path to the reference checkout> python tests/golden/make_golden.py
"""
from __future__ import annotations

import importlib
import math
import os
import random
import sys
import types
from pathlib import Path
from unittest import mock

import numpy as np

OUT = Path(__file__).resolve().parent
REF: Path | None = None


def _reference_root() -> Path:
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NESO_REFERENCE")
    if not arg:
        raise SystemExit("name the reference checkout: NESO_REFERENCE=<path> or the first argument")
    root = Path(arg)
    if not (root / "tests" / "test_rel_pos_fa2.py").exists():
        raise SystemExit(f"{root} does not look like the reference checkout (no tests/test_rel_pos_fa2.py)")
    return root


def _import_reference():
    metal = types.ModuleType("Metal")
    metal.MTLCreateSystemDefaultDevice = lambda: mock.MagicMock()
    sys.modules.setdefault("Metal", metal)
    for p in (REF / "src", REF / "tests"):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))
    relpos = importlib.import_module("test_rel_pos_fa2")
    quant = importlib.import_module("test_quantized_matmul")
    return relpos, quant


def relpos_case(relpos, T: int, d: int, nh: int) -> dict:
    """Inputs exactly as tests/test_rel_pos_fa2.py:314-330 draws them."""
    np.random.seed(42)
    scale = 1.0 / math.sqrt(d)
    Q = np.random.randn(nh, T, d).astype(np.float32) * 0.5
    K = np.random.randn(nh, T, d).astype(np.float32) * 0.5
    V = np.random.randn(nh, T, d).astype(np.float32) * 0.5
    K_rel = np.random.randn(nh, 2 * T - 1, d).astype(np.float32) * 0.5
    bias_u = np.random.randn(nh, d).astype(np.float32) * 0.1
    bias_v = np.random.randn(nh, d).astype(np.float32) * 0.1
    ref_out = relpos.reference_rel_pos_attention(
        Q.flatten().tolist(), K.flatten().tolist(), V.flatten().tolist(), K_rel.flatten().tolist(),
        bias_u.flatten().tolist(), bias_v.flatten().tolist(), T, d, nh, scale)
    Q_u, rel_bias = relpos.precompute_bias_and_qu(
        Q.flatten().tolist(), K_rel.flatten().tolist(), bias_u.flatten().tolist(), bias_v.flatten().tolist(),
        T, d, nh, scale)
    return dict(Q_u=Q_u.astype(np.float32), K=K, V=V, rel_bias=rel_bias.astype(np.float32),
                ref_out=np.asarray(ref_out, dtype=np.float64), T=T, d=d, nh=nh, scale=scale)


def fa2_case(relpos, N: int, d: int) -> dict:
    """Single-head FA2 inputs drawn as tests/test_flash_attention.py:263-272
    (random.seed(42), gauss(0, 0.5) for q, k, v). The expected output is the
    reference's own NumPy attention (reference_rel_pos_attention) with the
    relative terms switched off (K_rel = 0, bias_u = bias_v = 0), which is
    exactly softmax(Q K^T * scale) V."""
    random.seed(42)
    scale = 1.0 / math.sqrt(d)
    q = [random.gauss(0, 0.5) for _ in range(N * d)]
    k = [random.gauss(0, 0.5) for _ in range(N * d)]
    v = [random.gauss(0, 0.5) for _ in range(N * d)]
    zeros_rel = [0.0] * ((2 * N - 1) * d)
    zeros_b = [0.0] * d
    ref = relpos.reference_rel_pos_attention(q, k, v, zeros_rel, zeros_b, zeros_b, N, d, 1, scale)
    return dict(q=np.array(q, np.float32).reshape(N, d), k=np.array(k, np.float32).reshape(N, d),
                v=np.array(v, np.float32).reshape(N, d), ref_out=np.asarray(ref, np.float64).reshape(N, d),
                N=N, d=d, scale=scale)


def quant_case(quant, kind: str, M: int, N: int, K: int) -> dict:
    """Inputs drawn as tests/test_quantized_matmul.py:329-331 (w8a16, seed 42),
    :374-376 (w4a16 unpacked, seed 43) and :418-421 (scaled, seed 44); expected
    values from the reference's ref_* functions (:288-311)."""
    if kind == "w8a16":
        random.seed(42)
        a = [random.gauss(0, 0.5) for _ in range(M * K)]
        b = [random.randint(-128, 127) for _ in range(K * N)]
        ref = quant.ref_w8a16_matmul(a, b, M, N, K)
        s = None
    elif kind == "w4a16":
        random.seed(43)
        a = [random.gauss(0, 0.5) for _ in range(M * K)]
        b = [random.randint(-8, 7) for _ in range(K * N)]
        ref = quant.ref_w4a16_matmul(a, b, M, N, K)
        s = None
    elif kind == "w8a16_scaled":
        random.seed(44)
        a = [random.gauss(0, 0.5) for _ in range(M * K)]
        b = [random.randint(-128, 127) for _ in range(K * N)]
        s = [random.uniform(0.001, 0.1) for _ in range(N)]
        ref = quant.ref_w8a16_scaled_matmul(a, b, s, M, N, K)
    else:
        raise ValueError(kind)
    out = dict(a=np.array(a, np.float32).reshape(M, K), b=np.array(b, np.int8).reshape(K, N),
               ref=np.array(ref, np.float64).reshape(M, N), M=M, N=N, K=K)
    if s is not None:
        out["scale"] = np.array(s, np.float32)
    return out


def main() -> None:
    global REF
    REF = _reference_root()
    relpos, quant = _import_reference()
    cases = {
        # tests/test_rel_pos_fa2.py:435-437 configs (T, d, nh)
        "relpos_T32_d64_nh2": relpos_case(relpos, 32, 64, 2),
        "relpos_T64_d128_nh4": relpos_case(relpos, 64, 128, 4),
        # tests/test_flash_attention.py:398-448 sizes (N, d)
        "fa2_N128_d64": fa2_case(relpos, 128, 64),
        "fa2_N256_d128": fa2_case(relpos, 256, 128),
        # tests/test_quantized_matmul.py:531-580 sizes
        "w8a16_64": quant_case(quant, "w8a16", 64, 64, 64),
        "w4a16_64": quant_case(quant, "w4a16", 64, 64, 64),
        "w8a16_scaled_64": quant_case(quant, "w8a16_scaled", 64, 64, 64),
    }
    for name, arrays in cases.items():
        np.savez_compressed(OUT / f"{name}.npz", **arrays)
        print(f"wrote {name}.npz")


if __name__ == "__main__":
    main()
