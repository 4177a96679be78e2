"""SPK-side weight pre-packing (weight_layout TC_PANEL_F32X2).

The compiler stores the fp32 weights of tensor-core convs as the tcgen05
operand panel ([hi | lo][Npad][Kpad], K-major, k = (r, s, c)), so prepare on
the device uses them in place instead of repacking (reference format field
weight_layout, compiler/packager/spk_writer.py:35).  CPU checks here: the
panel arithmetic, what the package stores, and that the reader (and so the
oracle) recovers the exact OIHW weights; the GPU checks compare pre-packed and
runtime-packed packages bit for bit."""

from __future__ import annotations

import copy
import struct

import numpy as np
import pytest

from conftest import compile_pair, reference_outputs, seeded_input


def test_tc_panel_is_exact_and_rounds_tf32_to_nearest_ties_away():
    from spinnv2_b200.compiler.spk_writer import tc_panel, tc_panel_to_oihw

    rng = np.random.default_rng(3)
    w = rng.standard_normal((40, 12, 3, 3)).astype(np.float32)
    tie = np.float32(1.0 + 2.0 ** -11)  # halfway between two TF32 values
    w[0, 0, 0, 0], w[0, 0, 0, 1] = tie, -tie
    w[0, 0, 0, 2] = np.float32(1e-40)  # subnormal
    w[0, 0, 1, 0] = np.float32(3.0e38)
    panel = tc_panel(w)
    assert panel.shape == (2, 256, 128)
    hi = panel[0]
    assert not np.any(hi.view(np.uint32) & 0x1FFF)  # 10 mantissa bits
    assert hi[0, 0] == np.float32(1.0 + 2.0 ** -10) and hi[0, 12] == -np.float32(1.0 + 2.0 ** -10)  # ties away
    # k = (r * KW + s) * C + c: weight [m, c, r, s] sits at column (r * 3 + s) * 12 + c.
    m, c, r, s = 7, 5, 2, 1
    assert panel[0, m, (r * 3 + s) * 12 + c] + panel[1, m, (r * 3 + s) * 12 + c] == w[m, c, r, s]
    np.testing.assert_array_equal(tc_panel_to_oihw(panel, w.shape), w)
    assert not panel[:, 40:, :].any() and not panel[:, :, 108:].any()  # zero padding


def test_cuda_package_stores_panels_and_reader_recovers_weights():
    from spinnv2_b200.compiler import builders, pipeline
    from spinnv2_b200.compiler import spk_writer as W
    from spinnv2_b200.spk import read_spk

    spk = compile_pair("resnet50", 1, targets=("cuda_b200",))["cuda_b200"]
    pkg = read_spk(spk)
    graph = pipeline.fuse(builders.build_config("resnet50", 1))
    convs = [n for n in pkg.nodes if n.op_type == "Conv"]
    panels = pkg.panel_weights
    assert len(panels) == len(convs) - 1  # all but the 3-channel first conv
    for n in convs:
        t = pkg.tensors[n.inputs[1]]
        m, c, kh, kw = t.shape
        want = graph.tensors[graph.nodes[n.id].inputs[1]].array()
        if n.inputs[1] in panels:
            assert pkg.specs[n.kernel_spec_id].weight_layout == 2
            npad, kpad = -(-m // 256) * 256, -(-(c * kh * kw) // 32) * 32
            assert t.size_bytes == 2 * npad * kpad * 4
        else:
            assert t.size_bytes == want.nbytes
        np.testing.assert_array_equal(pkg.weight(n.inputs[1]), want)
    # The header's weight byte count is the stored (packed) total.
    assert pkg.header["weight_bytes"] == sum(pkg.tensors[t].size_bytes for t in range(len(pkg.tensors))
                                             if pkg.tensors[t].role_name == "weight")
    assert W.WEIGHT_LAYOUT_CODES["TC_PANEL_F32X2"] == 2


def test_prepacking_follows_the_profile_and_cpu_packages_keep_oihw():
    from spinnv2_b200.compiler import builders, pipeline
    from spinnv2_b200.compiler.profile import load_target_profile
    from spinnv2_b200.spk import read_spk

    graph = pipeline.fuse(builders.build_config("conv3x3_64_56", 2))
    prof = copy.deepcopy(load_target_profile("cuda_b200"))
    prof["weight_layouts"] = ["OIHW"]
    off = read_spk(pipeline.package(copy.deepcopy(graph), prof))
    on = read_spk(pipeline.package(copy.deepcopy(graph), "cuda_b200"))
    cpu = read_spk(pipeline.package(copy.deepcopy(graph), "cpu_generic_x86"))
    assert not off.panel_weights and not cpu.panel_weights and len(on.panel_weights) == 1
    wid = next(iter(on.panel_weights))
    np.testing.assert_array_equal(on.weight(wid), off.weight(wid))


def test_oracle_runs_prepacked_packages():
    """The CPU oracle reads weights through the package reader, so it runs a
    pre-packed CUDA package and agrees with the reference runtime."""
    from oracle import harness

    spk = compile_pair("conv3x3_64_56", 1)
    x = seeded_input((1, 64, 56, 56), seed=2)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out = harness.run_spk(spk["cuda_b200"], [x])[0][0]
    np.testing.assert_allclose(out, ref, atol=1e-3, rtol=1e-4)


def _package_pair(case: str, batch: int):
    from spinnv2_b200.compiler import builders, pipeline
    from spinnv2_b200.compiler.profile import load_target_profile

    graph = pipeline.fuse(builders.build_config(case, batch))
    prof = copy.deepcopy(load_target_profile("cuda_b200"))
    prof["weight_layouts"] = ["OIHW"]
    return pipeline.package(copy.deepcopy(graph), "cuda_b200"), pipeline.package(copy.deepcopy(graph), prof)


@pytest.mark.gpu
@pytest.mark.parametrize("case,batch", [("resnet50", 2), ("conv3x3_256_14", 1), ("conv1x1_2048_512_7", 32)])
@pytest.mark.parametrize("math", ["3xtf32", "tf32"])
def test_prepacked_and_runtime_packed_panels_give_identical_outputs(gpu, case, batch, math):
    from spinnv2_b200.runtime import MATH_3XTF32, MATH_TF32, Runtime
    from spinnv2_b200.spk import read_spk

    packed, raw = _package_pair(case, batch)
    x = seeded_input(read_spk(packed).inputs[0].shape, seed=19)
    mode = MATH_3XTF32 if math == "3xtf32" else MATH_TF32
    outs = []
    for spk, tag in ((packed, "_prepacked"), (raw, None)):
        with Runtime(spk, device=0, math_mode=mode) as rt:
            outs.append(rt.run(x)[0])
            variants = [rt.node_variant(n.id) for n in rt.package.nodes if n.op_type == "Conv"]
        if tag:
            assert sum(tag in v for v in variants) >= len(variants) - (1 if case == "resnet50" else 0), variants
        else:
            assert not any("_prepacked" in v for v in variants), variants
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.gpu
def test_prepacked_weights_on_the_cuda_core_path(gpu):
    """FP32 math mode runs the CUDA-core conv, which unpacks the stored panel
    to OIHW at prepare."""
    from spinnv2_b200.runtime import MATH_FP32, Runtime

    spk = compile_pair("conv3x3_128_28", 2)
    x = seeded_input((2, 128, 28, 28), seed=23)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    with Runtime(spk["cuda_b200"], device=0, math_mode=MATH_FP32) as rt:
        out = rt.run(x)[0]
        variant = rt.node_variant(next(n.id for n in rt.package.nodes if n.op_type == "Conv"))
    assert variant.startswith("simt_fp32"), variant
    np.testing.assert_allclose(out, ref, atol=1e-3, rtol=1e-4)
