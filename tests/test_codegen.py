"""Generated-C deployment path: spinnv2_b200.compiler.c_codegen emits the
static wrapper (embedded package, <sym>_init/_run/_run_checked/_run_multi/
_verify_checksum/_free) that a deployment links against a runtime library.

The same generator output is compiled with gcc and linked (a) against the
reference SPINNV2 CPU runtime (oracle/_ref/libspkv2_ref.so) for a CPU-profile
package, where it must reproduce the reference outputs bit for bit, and (b)
against this repository's libspkv2_runtime.so for a cuda_b200 package, where
it runs on the B200 (gpu marker) and must match the reference within the
fp32 tolerance max-abs 1e-3, rel 1e-4.  tests/c/gen_main.c is the driver."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import REPO, compile_pair, reference_outputs, seeded_input

DRIVER = REPO / "tests" / "c" / "gen_main.c"


def _gcc() -> str:
    cc = shutil.which("gcc-13") or shutil.which("gcc")
    if not cc:
        pytest.skip("no host C compiler")
    return cc


def _build(spk: bytes, out: Path, lib_dir: Path, lib: str) -> Path:
    from spinnv2_b200.compiler import c_codegen

    c_codegen.generate(spk, "model", out)
    exe = out / "run"
    cmd = [_gcc(), "-std=c99", "-O2", "-Wall", "-Werror", "-I", str(REPO / "include"), "-I", str(out), str(DRIVER),
           str(out / "model.c"), "-L", str(lib_dir), f"-l{lib}", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def _run_all(exe: Path, xs: list, outs: list, tmp: Path, runs: int = 3) -> list:
    """Runs the driver on the inputs `xs` (written back to back); `outs` is
    the (shape, dtype) of each output, read back to back."""
    fin, fout = tmp / "in.bin", tmp / "out.bin"
    fin.write_bytes(b"".join(np.ascontiguousarray(x).tobytes() for x in xs))
    res = subprocess.run([str(exe), str(fin), str(fout), str(runs)], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr
    raw, got, off = fout.read_bytes(), [], 0
    for shape, dt in outs:
        n = int(np.prod(shape)) * np.dtype(dt).itemsize
        got.append(np.frombuffer(raw[off:off + n], dtype=dt).reshape(shape))
        off += n
    assert off == len(raw)
    return got


def _run(exe: Path, x: np.ndarray, out_shape, tmp: Path, runs: int = 3) -> np.ndarray:
    return _run_all(exe, [x.astype(np.float32)], [(out_shape, np.float32)], tmp, runs)[0]


def test_header_macros_and_arenas(built):
    from spinnv2_b200.compiler import c_codegen
    from spinnv2_b200.spk import read_spk

    spk = compile_pair("lenet5", 1)
    cpu = c_codegen.header_text("lenet", spk["cpu_generic_x86"])
    gpu = c_codegen.header_text("lenet", spk["cuda_b200"])
    pkg = read_spk(spk["cpu_generic_x86"])
    assert f"#define LENET_INPUT_SIZE_0 ((size_t){pkg.inputs[0].size_bytes}u)" in cpu
    assert f"#define LENET_ACTIVATION_ARENA_SIZE ((size_t){pkg.header['activation_arena_bytes']}u)" in cpu
    assert "#define LENET_HOST_ARENAS 1" in cpu
    # Device packages: the runtime owns the device arenas; no host arena is reserved.
    assert "#define LENET_HOST_ARENAS 0" in gpu and "#define LENET_ACTIVATION_ARENA_SIZE ((size_t)0u)" in gpu
    with pytest.raises(ValueError):
        c_codegen.header_text("1bad", spk["cuda_b200"])


def test_generated_c_on_reference_runtime_matches_reference(built, tmp_path):
    from oracle import REF_LIB

    spk = compile_pair("lenet5", 1)
    exe = _build(spk["cpu_generic_x86"], tmp_path, Path(REF_LIB).parent, "spkv2_ref")
    x = seeded_input((1, 1, 28, 28), "uniform")
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    np.testing.assert_array_equal(_run(exe, x, ref.shape, tmp_path), ref)


@pytest.mark.parametrize("case", ["gather_input", "topk_ties"])
def test_generated_c_run_multi_on_reference_runtime(built, tmp_path, case):
    """Packages with two inputs (Gather with runtime indices) or two outputs
    (TopK values and indices) go through <sym>_run_multi, with the size
    arrays taken from the header's <SYM>_INPUT_SIZES / <SYM>_OUTPUT_SIZES."""
    from oracle import REF_LIB
    from spinnv2_b200.spk import read_spk
    from test_ops import op_inputs

    spk = compile_pair(f"op_{case}", 2)
    pkg = read_spk(spk["cpu_generic_x86"])
    assert len(pkg.inputs) + len(pkg.outputs) == 3
    exe = _build(spk["cpu_generic_x86"], tmp_path, Path(REF_LIB).parent, "spkv2_ref")
    ins = op_inputs(pkg)
    ref = reference_outputs(spk["cpu_generic_x86"], ins)
    got = _run_all(exe, ins, [(tuple(t.shape), t.np_dtype) for t in pkg.outputs], tmp_path)
    for g, r in zip(got, ref):
        np.testing.assert_array_equal(g, r)


def test_generated_c_links_against_cuda_runtime(built, tmp_path):
    from spinnv2_b200.runtime import LIB_PATH

    spk = compile_pair("lenet5", 1)
    exe = _build(spk["cuda_b200"], tmp_path, LIB_PATH.parent, "spkv2_runtime")
    assert exe.exists()


@pytest.mark.gpu
@pytest.mark.parametrize("name,shape,kind", [("lenet5", (1, 1, 28, 28), "uniform"),
                                             ("conv3x3_64_56", (2, 64, 56, 56), "normal")])
def test_generated_c_on_cuda_runtime_matches_reference(gpu, tmp_path, name, shape, kind):
    from spinnv2_b200.runtime import LIB_PATH

    spk = compile_pair(name, shape[0])
    exe = _build(spk["cuda_b200"], tmp_path, LIB_PATH.parent, "spkv2_runtime")
    x = seeded_input(shape, kind)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    np.testing.assert_allclose(_run(exe, x, ref.shape, tmp_path), ref, atol=1e-3, rtol=1e-4)


@pytest.mark.gpu
def test_generated_c_run_multi_on_cuda_runtime(gpu, tmp_path):
    """TopK (two outputs, values and int indices) through <sym>_run_multi on
    the B200: bit-exact with the reference (the scores come from one Mul and
    one Mod, single IEEE operations, so the selection sees the same keys)."""
    from spinnv2_b200.runtime import LIB_PATH
    from spinnv2_b200.spk import read_spk
    from test_ops import op_inputs

    spk = compile_pair("op_topk_ties", 2)
    pkg = read_spk(spk["cpu_generic_x86"])
    exe = _build(spk["cuda_b200"], tmp_path, LIB_PATH.parent, "spkv2_runtime")
    ins = op_inputs(pkg)
    ref = reference_outputs(spk["cpu_generic_x86"], ins)
    got = _run_all(exe, ins, [(tuple(t.shape), t.np_dtype) for t in pkg.outputs], tmp_path)
    for g, r in zip(got, ref):
        np.testing.assert_array_equal(g, r)
