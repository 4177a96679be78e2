"""Shared fixtures.  `-m gpu` tests need a B200 and the built runtime; the rest
run on the CPU (they may load the library: loading needs no GPU)."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and the built CUDA runtime")


def _ensure_built():
    from spinnv2_b200.runtime import LIB_PATH
    from oracle import ORACLE_LIB, REF_LIB

    if not LIB_PATH.exists() or not ORACLE_LIB.exists() or not REF_LIB.exists():
        import __graft_entry__

        __graft_entry__.build()


@pytest.fixture(scope="session")
def built():
    _ensure_built()
    return True


@pytest.fixture(scope="session")
def gpu(built):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    return 0


def compile_pair(name: str, batch: int, targets=("cuda_b200", "cpu_generic_x86"), **kw) -> dict:
    from spinnv2_b200.compiler import pipeline

    return pipeline.compile_config(name, batch, targets=targets, **kw)


def seeded_input(shape, kind: str = "normal", seed: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "uniform":
        return rng.random(shape, dtype=np.float32)
    return rng.standard_normal(shape, dtype=np.float32)


def reference_outputs(spk_cpu: bytes, inputs: list[np.ndarray]) -> list[np.ndarray]:
    from oracle import refrt
    from spinnv2_b200.spk import read_spk

    pkg = read_spk(spk_cpu)
    return refrt.run_reference(spk_cpu, inputs, [(tuple(t.shape), t.np_dtype) for t in pkg.outputs])


def compile_with_outputs(name: str, batch: int, pick, targets=("cuda_b200", "cpu_generic_x86")) -> dict:
    """Config `name` at `batch`, fused once, with extra graph outputs: the
    tensor ids pick(graph) returns (intermediates such as the pre-softmax
    logits) are appended to the graph's outputs, so the reference CPU runtime
    reports them too.  The convolutions and their plans are the config's."""
    import copy

    from spinnv2_b200.compiler import builders, pipeline

    graph = pipeline.fuse(builders.build_config(name, batch))
    from spinnv2_b200.compiler.ir import ROLE_OUTPUT

    extra = [t for t in pick(graph) if t not in graph.outputs]
    for t in extra:
        graph.tensors[t].role = ROLE_OUTPUT
    graph.outputs = list(graph.outputs) + extra
    return {t: pipeline.package(copy.deepcopy(graph), t) for t in targets}


def gemm_output(graph) -> list[int]:
    return [next(n for n in graph.nodes if n.op_type == "Gemm").outputs[0]]
