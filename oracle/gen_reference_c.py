"""Generate C with the REFERENCE compiler's code generator (test
infrastructure, run at build time where the reference tree is available).

    python oracle/gen_reference_c.py <reference_root> <out_dir>

Packages LeNet-5 (batch 1) for the x86 CPU profile and for the cuda_b200
profile with this repository's compiler, then runs the reference generator
(reference compiler/codegen/c_codegen.py:98-137, `generate_c_from_spk`:
model.h, model.c with the package embedded as a byte array and static
host arenas, and main_test.c) on each package.  The Makefile compiles the
generated files unchanged against include/ and libspkv2_runtime.so (and,
for comparison, against the reference runtime); tests/test_dropin.py runs
the binaries on the GPU.  Outputs go to <out_dir>/<profile>/; nothing here
is committed.
"""

from __future__ import annotations

import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def main() -> None:
    ref_root, out_dir = Path(sys.argv[1]), Path(sys.argv[2])
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(ref_root))
    from compiler.codegen.c_codegen import generate_c_from_spk  # reference generator

    from spinnv2_b200.compiler import pipeline

    spks = pipeline.compile_config("lenet5", 1, targets=("cpu_generic_x86", "cuda_b200"))
    for profile, data in spks.items():
        d = out_dir / profile
        d.mkdir(parents=True, exist_ok=True)
        (d / "lenet5.spk").write_bytes(data)
        generate_c_from_spk(d / "lenet5.spk", d, name="model", runtime_dir=ref_root / "runtime")
        print(d)


if __name__ == "__main__":
    main()
