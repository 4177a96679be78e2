"""Op coverage on the CPU: the numpy restatement of every runtime op outside
the five configs (MatMul, Clip, LeakyRelu, AveragePool, GlobalAveragePool,
Mod, Sub, Div, Transpose, Tile, Slice, Gather, Unsqueeze) is pinned against
the reference SPINNV2 runtime (oracle/_ref, built from the reference's own
sources) on seeded single-op graphs, and every such graph compiles for the
CUDA target with a CUDA spec (no CPU fallback token) for each node."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import compile_pair, reference_outputs, seeded_input

GATHER_INDICES = np.array([6, -1, 0, 3], dtype=np.float32)


def op_inputs(pkg):
    """Seeded inputs of an op-coverage package (the index input of
    gather_input gets fixed in-range indices, one of them negative)."""
    return [GATHER_INDICES if t.name == "indices" else seeded_input(tuple(t.shape)) for t in pkg.inputs]


def _case_ids():
    from spinnv2_b200.compiler.builders import OP_CASES

    return list(OP_CASES)


@pytest.mark.parametrize("case", _case_ids())
def test_oracle_matches_reference_runtime_on_op(built, case):
    from oracle import harness
    from spinnv2_b200.spk import read_spk

    spk = compile_pair(f"op_{case}", 2)
    pkg = read_spk(spk["cpu_generic_x86"])
    ins = op_inputs(pkg)
    ref = reference_outputs(spk["cpu_generic_x86"], ins)
    got, _ = harness.run_spk(spk["cuda_b200"], ins)
    for r, g in zip(ref, got):
        np.testing.assert_allclose(g, r, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("case", _case_ids())
def test_op_graph_compiles_to_cuda_specs_only(case):
    from spinnv2_b200.spk import read_spk

    pkg = read_spk(compile_pair(f"op_{case}", 2, targets=("cuda_b200",))["cuda_b200"])
    assert pkg.specs, "the CUDA package carries kernel specs"
    assert all(s.backend == "delegate" for s in pkg.specs)
    assert len(pkg.specs) == len(pkg.nodes)  # no reference fallback spec was emitted
