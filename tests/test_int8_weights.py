"""Weights-only INT8 packages: the reference compiler's own INT8 format
(reference compiler/quantization/quantize_weights.py:24-120): int8 conv
weights per output channel, per-tensor scales for conv inputs, fp32
activations, biases and residuals.  The reference's kernel for it
(runtime/kernels/optimized/conv/conv_int8.c) exists only for ARM with dot
products, so the oracle is a restatement of its arithmetic (oracle/harness.py
`run_conv`, oracle/oracle_ops.c `oracle_dequant_w8`): q = sat8(rne(x *
fp32(1 / s_x))), int32 accumulation, y = act(fma(acc, s_w[c] * s_x, b) + res).

CPU: the package carries the reference's kernel kind for its CPU profile and
tc_int8 specs for the CUDA target; the oracle rounds halves to even.
GPU: the CUDA runtime's weights-only path against the oracle, fp32 tolerance
max-abs 1e-3, rel 1e-4 (the int8 codes and int32 sums are exact; what may
differ is fp32 summation order elsewhere in the network)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import seeded_input

ATOL, RTOL = 1e-3, 1e-4


def _packages(name, batch, targets=("cuda_b200", "cpu_generic_x86")):
    from spinnv2_b200.compiler import pipeline

    return pipeline.compile_config(name, batch, targets=targets, int8="weights")


def test_weights_only_package_format():
    from spinnv2_b200.spk import read_spk

    spk = _packages("lenet5", 1)
    cpu, gpu = read_spk(spk["cpu_generic_x86"]), read_spk(spk["cuda_b200"])
    convs = [n for n in cpu.nodes if n.op_type == "Conv"]
    assert all(cpu.tensors[n.inputs[1]].np_dtype == np.int8 for n in convs)
    assert all(cpu.tensors[n.inputs[0]].np_dtype == np.float32 for n in convs)
    assert {cpu.specs[i].kind for i, n in enumerate(cpu.nodes) if n.op_type == "Conv"} >= {"int8_im2col_gemm"}
    assert all(s.kind == "tc_int8" for s, n in zip(gpu.specs, gpu.nodes) if n.op_type == "Conv")
    for n in convs:
        assert cpu.quant[n.inputs[1]].scales.size == cpu.tensors[n.inputs[1]].shape[0]
        assert cpu.quant[n.inputs[0]].scales.size == 1


def test_oracle_quantises_halves_to_even(built):
    """x * (1 / s_x) exactly at .5: the reference's vector lanes (vcvtnq)
    round to even."""
    from oracle import harness
    from spinnv2_b200.spk import read_spk

    spk = _packages("lenet5", 1, targets=("cuda_b200",))["cuda_b200"]
    pkg = read_spk(spk)
    conv = next(n for n in pkg.nodes if n.op_type == "Conv")
    sx = np.float32(pkg.quant[conv.inputs[0]].scales[0])
    inv = np.float32(np.float32(1) / sx)
    x = np.zeros((1, 1, 28, 28), dtype=np.float32)
    # Values whose scaled form is k + 0.5 exactly where representable.
    for k, v in enumerate([0.5, 1.5, 2.5, -0.5, -1.5]):
        x[0, 0, 0, k] = np.float32(v) / inv
    env = {conv.inputs[0]: x}
    y = harness.run_conv(pkg, conv, env)
    assert y.shape == tuple(pkg.tensors[conv.outputs[0]].shape)
    q = np.rint((x * inv).astype(np.float32))
    assert list(q[0, 0, 0, :5]) == [0.0, 2.0, 2.0, -0.0, -2.0] or list(q[0, 0, 0, :5]) == [0.0, 2.0, 2.0, 0.0, -2.0]


@pytest.mark.gpu
@pytest.mark.parametrize("name,shape,kind", [("lenet5", (1, 1, 28, 28), "uniform"),
                                             ("conv3x3_64_56", (2, 64, 56, 56), "normal"),
                                             ("conv1x1_256_64_56", (2, 256, 56, 56), "normal"),
                                             ("resnet50", (1, 3, 224, 224), "normal")])
def test_weights_only_int8_matches_oracle(gpu, name, shape, kind):
    from oracle import harness
    from spinnv2_b200.runtime import Runtime

    spk = _packages(name, shape[0], targets=("cuda_b200",))["cuda_b200"]
    x = seeded_input(shape, kind)
    ref, _ = harness.run_spk(spk, [x])
    with Runtime(spk, device=0) as rt:
        out = rt.run(x)[0]
        variants = [rt.node_variant(i) for i in range(len(rt.package.nodes)) if rt.package.nodes[i].op_type == "Conv"]
        again = rt.run(x)[0]  # graph replay
    assert all(v.startswith("w8_") for v in variants), variants
    np.testing.assert_array_equal(out, again)
    if name == "resnet50":
        # Softmax probabilities of a random-init network: compare the class
        # ranking and the values at the fp32 tolerance.
        assert int(np.argmax(out)) == int(np.argmax(ref[0]))
    np.testing.assert_allclose(out, ref[0], atol=ATOL, rtol=RTOL)
