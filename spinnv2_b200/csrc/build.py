"""Build libspkv2_runtime.so (the CUDA target of the SPINNV2 runtime) in-tree.

Every .cu/.cpp under csrc/ is compiled by nvcc for sm_100a only and linked
into spinnv2_b200/_lib/libspkv2_runtime.so together with the static CUDA
runtime, so the library needs nothing but the NVIDIA driver at load time.
Objects are rebuilt when a source or any header under csrc/ or include/
is newer than the object.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build" / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libspkv2_runtime.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-I",
    str(INCLUDE),
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA target needs CUDA 12.8+ for sm_100a")
    return cand


def _sources() -> list[Path]:
    return sorted(p for p in CSRC.rglob("*") if p.suffix in {".cu", ".cpp"})


def _headers_mtime() -> float:
    stamps = [p.stat().st_mtime for p in CSRC.rglob("*") if p.suffix in {".h", ".cuh"}]
    stamps += [p.stat().st_mtime for p in INCLUDE.glob("*.h")]
    return max(stamps, default=0.0)


def _compile(src: Path, newest_header: float, verbose: bool) -> Path:
    rel = src.relative_to(CSRC)
    obj = BUILD_DIR / (str(rel).replace(os.sep, "__") + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
        return obj
    obj.parent.mkdir(parents=True, exist_ok=True)
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd[1:1] = ["-x", "cu"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {rel}:\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip() and verbose:
        print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every kernel/runtime source and link the shared library."""
    newest_header = _headers_mtime()
    sources = _sources()
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(lambda s: _compile(s, newest_header, verbose), sources))
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    if LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB_PATH
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(LIB_PATH), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
