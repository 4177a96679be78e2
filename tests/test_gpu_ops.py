"""GPU parity for the runtime ops outside the five configs: each seeded
single-op graph (x -> Add -> OP -> Add -> y) runs through the C-ABI runtime
on the B200 and is compared with the reference SPINNV2 CPU runtime
(oracle/_ref) on the same package graph and inputs.

Data movement and single IEEE operations (Clip, LeakyRelu, Mod, Sub, Div,
Transpose, Tile, Slice, Gather, Unsqueeze and the surrounding Adds) must be
bit-exact; MatMul and the average pools sum in a different order than the
reference's sequential loops and are held to the fp32 tolerance of the
parity suite, max-abs 1e-3 and rel 1e-4 (np.allclose(gpu, ref, atol=1e-3,
rtol=1e-4))."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import compile_pair, reference_outputs
from test_ops import GATHER_INDICES, _case_ids, op_inputs

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4
SUMMING = {"matmul", "matmul_bcast", "avgpool", "globalavgpool", "softmax_channels"}
SPKV2_ERR_DEVICE_STATUS = -47
INDEX_RANGE_CODE = 10


@pytest.mark.parametrize("case", _case_ids())
def test_op_matches_reference(gpu, case):
    from spinnv2_b200.runtime import LAYOUT_NHWC, Runtime
    from spinnv2_b200.spk import read_spk

    spk = compile_pair(f"op_{case}", 2)
    pkg = read_spk(spk["cuda_b200"])
    ins = op_inputs(pkg)
    ref = reference_outputs(spk["cpu_generic_x86"], ins)
    with Runtime(spk["cuda_b200"], device=0) as rt:
        first = rt.run(*ins)
        second = rt.run(*ins)  # graph replay
        op = pkg.nodes[1]
        variant = rt.node_variant(1)
        # The op under test reads an arena activation, NHWC where it is a
        # rank-4 tensor with C > 1 and H*W > 1.
        x = pkg.tensors[op.inputs[0]]
        nhwc = len(x.shape) == 4 and x.shape[1] > 1 and x.shape[2] * x.shape[3] > 1
        if nhwc:
            assert rt.tensor_layout(op.inputs[0]) == LAYOUT_NHWC
    assert variant, "the node has a CUDA kernel"
    for r, a, b in zip(ref, first, second):
        np.testing.assert_array_equal(a, b)
        if case in SUMMING:
            np.testing.assert_allclose(a, r, atol=ATOL, rtol=RTOL)
        else:
            np.testing.assert_array_equal(a, r)


def test_gather_out_of_range_index_reports_and_context_stays_usable(gpu):
    """An index outside [-dim, dim) after wrapping is caught by the kernel's
    own bounds check before any load: the element is written as 0, the run
    returns SPKV2_ERR_DEVICE_STATUS with device code 10, and the next run
    with valid indices is correct."""
    from spinnv2_b200.runtime import Runtime, Spkv2Error
    from spinnv2_b200.spk import read_spk

    spk = compile_pair("op_gather_input", 2)
    pkg = read_spk(spk["cuda_b200"])
    ins = op_inputs(pkg)
    ref = reference_outputs(spk["cpu_generic_x86"], ins)
    bad = [ins[0], np.array([6, 7, -8, 1], dtype=np.float32)]  # axis size 7: 7 and -8 are out of range
    assert np.array_equal(ins[1], GATHER_INDICES)
    with Runtime(spk["cuda_b200"], device=0) as rt:
        np.testing.assert_array_equal(rt.run(*ins)[0], ref[0])
        with pytest.raises(Spkv2Error) as err:
            rt.run(*bad)
        assert err.value.code == SPKV2_ERR_DEVICE_STATUS
        assert rt.lib.spkv2_cuda_last_device_code(rt.ctx) == INDEX_RANGE_CODE
        np.testing.assert_array_equal(rt.run(*ins)[0], ref[0])
