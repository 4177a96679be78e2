"""The reference ctypes driver against this library, on the CPU.

research/reliability/runtime_driver.py (the reference's reliability
driver) is imported from the reference tree where it is present and
pointed, unchanged, at libspkv2_runtime.so: every symbol it binds resolves
with its argtypes, a cuda_b200 package loads, and prepare, which needs an
sm_100 device, fails with this target's code -42 through the driver's own
error path.  (The GPU tests never read the reference tree; the same calling
sequence runs on the B200 through spinnv2_b200.runtime.RuntimeDriver.)
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

from conftest import compile_pair


def _reference_driver():
    import __graft_entry__

    root = __graft_entry__.reference_root()
    if root is None:
        return None
    path = Path(root) / "research" / "reliability" / "runtime_driver.py"
    return path if path.exists() else None


def test_reference_ctypes_driver_binds_the_cuda_library(built, tmp_path):
    import torch

    from spinnv2_b200.runtime import LIB_PATH

    path = _reference_driver()
    if path is None:
        pytest.skip("reference tree not present")
    if torch.cuda.is_available():
        pytest.skip("checks the no-device path; on a GPU the runtime's own RuntimeDriver test runs")
    import sys

    root = str(path.parents[2])  # the driver imports research.reliability.* from the tree's root
    sys.path.insert(0, root)
    try:
        spec = importlib.util.spec_from_file_location("ref_runtime_driver", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        sys.path.remove(root)
    spk = compile_pair("lenet5", 1)
    (tmp_path / "m.spk").write_bytes(spk["cuda_b200"])
    with pytest.raises(Exception, match="-42"):
        mod.RuntimeDriver(LIB_PATH, tmp_path / "m.spk")
