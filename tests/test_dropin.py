"""The drop-in claim, shown with the reference's own callers.

oracle/Makefile (target `dropin`, run by the build where the reference tree
is present) compiles, UNCHANGED, against this repository's include/ and
libspkv2_runtime.so:

- the reference command-line tools runtime/tools/spkv2_run.c (load_file ->
  prepare -> set_input -> run -> get_output) and spkv2_bench.c (its
  warm-up / timed-runs protocol and JSON report, all outputs dumped);
- the reference code generator's output (compiler/codegen/c_codegen.py
  `generate_c_from_spk`: model.c with the package embedded and static host
  arenas, plus main_test.c), for a LeNet-5 package of the x86 CPU profile
  and of the cuda_b200 profile; the same generated C is also linked against
  the reference CPU runtime.

These tests run those binaries on the B200 and compare their output files
with the reference CPU runtime's results (fp32 tolerance atol 1e-3, rtol
1e-4, element-wise).
"""

from __future__ import annotations

import json
import subprocess

import numpy as np
import pytest

from conftest import REPO, compile_pair, reference_outputs, seeded_input

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4
REF_DIR = REPO / "oracle" / "_ref"


def _binary(name: str):
    path = REF_DIR / name
    if not path.exists():
        pytest.fail(f"{path} was not built (oracle/Makefile target dropin, run by __graft_entry__.build())")
    return path


def _run(cmd, timeout=300) -> subprocess.CompletedProcess:
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True, timeout=timeout)
    assert res.returncode == 0, (cmd, res.returncode, res.stdout[-2000:], res.stderr[-2000:])
    return res


@pytest.mark.parametrize("config,batch,kind", [("lenet5", 1, "uniform"), ("resnet50", 2, "normal"),
                                               ("yolo_style", 1, "uniform")])
def test_reference_spkv2_run_tool_on_the_cuda_library(gpu, tmp_path, config, batch, kind):
    from spinnv2_b200.spk import read_spk

    spk = compile_pair(config, batch)
    pkg = read_spk(spk["cuda_b200"])
    x = seeded_input(pkg.inputs[0].shape, kind, seed=31)
    (tmp_path / "m.spk").write_bytes(spk["cuda_b200"])
    x.tofile(tmp_path / "in.bin")
    _run([_binary("spkv2_run_cuda"), tmp_path / "m.spk", tmp_path / "in.bin", tmp_path / "out.bin"])
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out = np.fromfile(tmp_path / "out.bin", dtype=ref.dtype).reshape(ref.shape)
    np.testing.assert_allclose(out, ref, atol=ATOL, rtol=RTOL)


def test_reference_spkv2_bench_tool_on_the_cuda_library(gpu, tmp_path):
    """spkv2_bench's own protocol (warm-up, timed spkv2_run calls, p50/p90)
    on the CUDA library, and its dump of every output after the last run."""
    from spinnv2_b200.spk import read_spk

    spk = compile_pair("yolo_style", 1)
    pkg = read_spk(spk["cuda_b200"])
    x = seeded_input(pkg.inputs[0].shape, "uniform", seed=37)
    (tmp_path / "m.spk").write_bytes(spk["cuda_b200"])
    x.tofile(tmp_path / "in.bin")
    res = _run([_binary("spkv2_bench_cuda"), tmp_path / "m.spk", tmp_path / "in.bin", tmp_path / "out.bin",
                "--warmup", "3", "--runs", "20"])
    report = json.loads(res.stdout[res.stdout.index("{"):res.stdout.index("}") + 1])
    assert report["runs"] == 20 and 0 < report["p50_ms"] <= report["max_ms"]
    print("spkv2_bench on the CUDA library, yolo_style bs1:", report)
    refs = reference_outputs(spk["cpu_generic_x86"], [x])
    raw = np.fromfile(tmp_path / "out.bin", dtype=np.uint8)
    off = 0
    for r in refs:
        n = r.nbytes
        got = raw[off:off + n].view(r.dtype).reshape(r.shape)
        off += n
        if r is refs[0]:  # top-300 scores
            np.testing.assert_allclose(got, r, atol=ATOL, rtol=RTOL)
    assert off == raw.size


@pytest.mark.parametrize("binary", ["main_test_cuda_b200", "main_test_cpu_on_cuda"])
def test_reference_generated_c_on_the_cuda_library(gpu, tmp_path, binary):
    """The reference generator's model.c + main_test.c (LeNet-5, package
    embedded, static host arenas) linked against the CUDA library, against
    the same generated C linked against the reference CPU runtime."""
    x = seeded_input((1, 1, 28, 28), "uniform", seed=41)
    x.tofile(tmp_path / "in.bin")
    _run([_binary(f"gen/{binary}"), tmp_path / "in.bin", tmp_path / "out_gpu.bin"])
    _run([_binary("gen/main_test_cpu_on_ref"), tmp_path / "in.bin", tmp_path / "out_ref.bin"])
    out = np.fromfile(tmp_path / "out_gpu.bin", dtype=np.float32)
    ref = np.fromfile(tmp_path / "out_ref.bin", dtype=np.float32)
    assert out.size == ref.size == 10
    np.testing.assert_allclose(out, ref, atol=ATOL, rtol=RTOL)

