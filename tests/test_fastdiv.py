"""The tensor-core conv kernels, the split-K reduce and the reductions compute
tile, pixel and schedule coordinates with 32-bit multiply-shift divisions
(spkv2::FastDiv in csrc/kernels/common.cuh).  This CPU test compiles the
host branch of the same arithmetic with nvcc and checks it against integer
division over every divisor below 4097, the named networks' pixel, tile and
K-step counts, powers of two and their neighbours and seeded random
divisors, at edge and seeded random numerators (tests/c/fastdiv_check.cu)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _nvcc() -> str | None:
    return shutil.which("nvcc") or (
        "/usr/local/cuda/bin/nvcc" if Path("/usr/local/cuda/bin/nvcc").exists() else None)


def test_fastdiv_matches_integer_division(tmp_path):
    nvcc = _nvcc()
    if nvcc is None:
        pytest.skip("nvcc not found")
    exe = tmp_path / "fastdiv_check"
    cmd = [nvcc, "-std=c++17", "-O2", "--expt-relaxed-constexpr", "-Wno-deprecated-gpu-targets",
           "-I", str(REPO / "include"), "-I", str(REPO / "spinnv2_b200" / "csrc" / "kernels"),
           "-I", str(REPO / "spinnv2_b200" / "csrc" / "runtime"),
           str(REPO / "tests" / "c" / "fastdiv_check.cu"), "-o", str(exe)]
    build = subprocess.run(cmd, capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.startswith("ok "), run.stdout
    assert int(run.stdout.split()[1]) > 10_000_000
