"""CPU checkers for the CUDA target - TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, as the checker and the timed CPU baseline; the product path
(spinnv2_b200, libspkv2_runtime.so) never does.

  refrt     ctypes driver of _ref/libspkv2_ref.so, the reference SPINNV2 C
            runtime compiled from its own sources by ./Makefile (`make ref`)
  harness   SPK interpreter on the CPU: numpy for the memory-bound ops, the C
            restatement in oracle_ops.c (`make oracle`) for Conv, including
            the INT8 requantisation contract the reference cannot run on x86
"""

from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
REF_LIB = ORACLE_DIR / "_ref" / "libspkv2_ref.so"
REF_BENCH = ORACLE_DIR / "_ref" / "spkv2_bench"
ORACLE_LIB = ORACLE_DIR / "_lib" / "liboracle.so"
