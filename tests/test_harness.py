"""The native harness (neso_b200/neso_harness), the C++ re-host of the
reference's Rust harness protocol (macos/harness.rs:201-365)."""
import subprocess
from pathlib import Path

import pytest

HARNESS = Path(__file__).resolve().parent.parent / "neso_b200" / "neso_harness"


def test_harness_built_and_prints_usage():
    assert HARNESS.exists(), "build with `python -m neso_b200.build`"
    r = subprocess.run([str(HARNESS)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2
    assert "usage: neso_harness <test|bench>" in r.stderr


@pytest.mark.gpu
def test_harness_known_answer_tests():
    r = subprocess.run([str(HARNESS), "test"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    for line in ("PASS vector_add (65537 elements, masked tail, bit-exact)",
                 "PASS scale (65537 elements, scalar argument, bit-exact)",
                 "PASS flash_attention_2 (f16, N=64, d=64"):
        assert line in r.stdout, r.stdout


@pytest.mark.gpu
def test_harness_bench_runs():
    r = subprocess.run([str(HARNESS), "bench"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "vector_add" in r.stdout and "flash_attn2 f16 N=2048" in r.stdout
