"""Conv attribute forms that the named models do not use, but SPINNV2's
reference conv accepts (reference runtime/kernels/reference/conv/conv.c:22-50):
grouped and depthwise convs, dilations, non-square kernels and strides, odd and
rectangular extents, and a bias with Relu fused.

CPU: the oracle restatement matches the reference runtime built from its own
sources, on these forms and on forty seeded random ones.  B200: the CUDA runtime (tensor-core path where it accepts the form,
the CUDA-core conv otherwise) matches the reference runtime within the fp32
tolerance of the parity suite, np.allclose(gpu, ref, atol=1e-3, rtol=1e-4),
eager and graph-replayed runs bit-identical."""

from __future__ import annotations

import copy

import numpy as np
import pytest

from conftest import reference_outputs

ATOL, RTOL = 1e-3, 1e-4

# name: (n, c, h, w, m, (kh, kw), (sh, sw), (pad_top, pad_left, pad_bottom, pad_right), (dh, dw), group, relu)
CASES = {
    "group2_3x3": (2, 16, 13, 11, 32, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 2, True),
    "depthwise_3x3_s2": (2, 32, 15, 15, 32, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), 32, False),
    "dilation2_3x3": (2, 32, 17, 17, 32, (3, 3), (1, 1), (2, 2, 2, 2), (2, 2), 1, True),
    "kernel_1x3": (1, 24, 9, 14, 40, (1, 3), (1, 1), (0, 1, 0, 1), (1, 1), 1, False),
    "kernel_3x1_s2x1": (2, 20, 12, 7, 36, (3, 1), (2, 1), (1, 0, 1, 0), (1, 1), 1, True),
    "kernel_5x5_s2_c3": (2, 3, 31, 29, 24, (5, 5), (2, 2), (2, 2, 2, 2), (1, 1), 1, True),
    "pad_asymmetric": (1, 32, 10, 10, 48, (3, 3), (1, 1), (0, 0, 1, 1), (1, 1), 1, False),
}


def _graph(case: str):
    from spinnv2_b200.compiler.ir import GraphBuilder

    n, c, h, w, m, (kh, kw), (sh, sw), pads, (dh, dw), group, relu = CASES[case]
    oh = (h + pads[0] + pads[2] - dh * (kh - 1) - 1) // sh + 1
    ow = (w + pads[1] + pads[3] - dw * (kw - 1) - 1) // sw + 1
    rng = np.random.default_rng(sum(map(ord, case)))
    b = GraphBuilder(f"geom_{case}")
    x = b.input("input", [n, c, h, w])
    # An Add before the conv keeps its input an internal (device-layout) tensor.
    x1 = b.op("Add", [x, b.weight("pre_c", np.array([0.125], np.float32))], [n, c, h, w])
    fan_in = (c // group) * kh * kw
    wt = (rng.standard_normal((m, c // group, kh, kw)) * np.sqrt(2.0 / fan_in)).astype(np.float32)
    bias = (rng.standard_normal(m) * 0.1).astype(np.float32)
    attrs = {"kernel_shape": [kh, kw], "strides": [sh, sw], "pads": list(pads), "dilations": [dh, dw],
             "group": group}
    y = b.op("Conv", [x1, b.weight("w", wt), b.weight("b", bias)], [n, m, oh, ow], attrs)
    if relu:
        y = b.op("Relu", [y], [n, m, oh, ow])
    b.mark_output(y)
    x_in = rng.standard_normal((n, c, h, w)).astype(np.float32)
    return b.graph, x_in


def _packages(case: str):
    from spinnv2_b200.compiler import pipeline

    graph, x = _graph(case)
    graph = pipeline.fuse(graph)
    return (pipeline.package(copy.deepcopy(graph), "cuda_b200"),
            pipeline.package(copy.deepcopy(graph), "cpu_generic_x86"), x)


@pytest.mark.parametrize("case", sorted(CASES))
def test_oracle_matches_reference_runtime_on_conv_form(built, case):
    from oracle import harness

    spk_gpu, spk_cpu, x = _packages(case)
    ref = reference_outputs(spk_cpu, [x])
    mine, _ = harness.run_spk(spk_gpu, [x])
    for r, o in zip(ref, mine):
        np.testing.assert_allclose(o, r, rtol=1e-5, atol=1e-5)


def _random_forms(count: int, seed: int):
    """Seeded random conv attribute forms: groups 1/2/4, 1-8 channels per
    group, kernels 1-5 per side, strides 1-3, dilations 1-2, each pad 0-2,
    extents 1-15."""
    rng = np.random.default_rng(seed)
    forms = []
    while len(forms) < count:
        group = int(rng.choice([1, 1, 2, 4]))
        c, m = group * int(rng.integers(1, 9)), group * int(rng.integers(1, 9))
        kh, kw = int(rng.integers(1, 6)), int(rng.integers(1, 6))
        sh, sw = int(rng.integers(1, 4)), int(rng.integers(1, 4))
        dh, dw = int(rng.integers(1, 3)), int(rng.integers(1, 3))
        pads = tuple(int(v) for v in rng.integers(0, 3, 4))
        h, w = int(rng.integers(1, 16)), int(rng.integers(1, 16))
        if (h + pads[0] + pads[2] - dh * (kh - 1) - 1) < 0 or (w + pads[1] + pads[3] - dw * (kw - 1) - 1) < 0:
            continue
        forms.append((int(rng.integers(1, 3)), c, h, w, m, (kh, kw), (sh, sw), pads, (dh, dw), group,
                      bool(rng.integers(0, 2))))
    return forms


def test_oracle_matches_reference_runtime_on_random_conv_forms(built):
    from oracle import harness

    for i, form in enumerate(_random_forms(40, 123)):
        CASES[f"random_{i}"] = form
        try:
            spk_gpu, spk_cpu, x = _packages(f"random_{i}")
        finally:
            del CASES[f"random_{i}"]
        ref = reference_outputs(spk_cpu, [x])[0]
        mine = harness.run_spk(spk_gpu, [x])[0][0]
        np.testing.assert_allclose(mine, ref, rtol=1e-5, atol=1e-5, err_msg=str(form))


@pytest.mark.gpu
@pytest.mark.parametrize("case", sorted(CASES))
def test_conv_form_matches_reference_on_b200(gpu, case):
    from spinnv2_b200.runtime import Runtime

    spk_gpu, spk_cpu, x = _packages(case)
    ref = reference_outputs(spk_cpu, [x])
    with Runtime(spk_gpu, device=0) as rt:
        eager = rt.run(x)
        replay = rt.run(x)
        conv = [i for i, nd in enumerate(rt.package.nodes) if nd.op_type == "Conv"]
        variant = rt.node_variant(conv[0])
    assert variant, "the conv has a CUDA kernel"
    for r, a, b in zip(ref, eager, replay):
        np.testing.assert_array_equal(a, b)
        err = np.abs(a - r)
        print(case, variant, "max abs", float(err.max()))
        np.testing.assert_allclose(a, r, atol=ATOL, rtol=RTOL)


def test_oracle_matches_reference_runtime_on_random_pool_forms(built):
    """MaxPool / AveragePool (reference runtime/kernels/reference/pool/
    maxpool.c, avgpool.c: pads[0], pads[1] at the top / left, the output
    extent from the output tensor, averages over the in-image taps) on
    seeded random kernels 1-5, strides 1-3, pads below the kernel and odd
    extents: the oracle matches the reference runtime."""
    import copy

    from oracle import harness
    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.compiler.ir import GraphBuilder

    rng = np.random.default_rng(7)
    checked = 0
    while checked < 40:
        op = str(rng.choice(["MaxPool", "AveragePool"]))
        kh, kw = int(rng.integers(1, 6)), int(rng.integers(1, 6))
        sh, sw = int(rng.integers(1, 4)), int(rng.integers(1, 4))
        p = [int(v) for v in rng.integers(0, 3, 4)]
        pads = [min(p[0], kh - 1), min(p[1], kw - 1), min(p[2], kh - 1), min(p[3], kw - 1)]
        n, c, h, w = (int(rng.integers(1, 3)), int(rng.integers(1, 10)), int(rng.integers(1, 14)),
                      int(rng.integers(1, 14)))
        oh, ow = (h + pads[0] + pads[2] - kh) // sh + 1, (w + pads[1] + pads[3] - kw) // sw + 1
        if oh < 1 or ow < 1:
            continue
        b = GraphBuilder(f"pool_form_{checked}")
        x = b.input("input", [n, c, h, w])
        x1 = b.op("Add", [x, b.weight("pre_c", np.array([0.125], np.float32))], [n, c, h, w])
        b.mark_output(b.op(op, [x1], [n, c, oh, ow], {"kernel_shape": [kh, kw], "strides": [sh, sw], "pads": pads}))
        graph = pipeline.fuse(b.graph)
        spk_gpu = pipeline.package(copy.deepcopy(graph), "cuda_b200")
        spk_cpu = pipeline.package(copy.deepcopy(graph), "cpu_generic_x86")
        xin = rng.standard_normal((n, c, h, w)).astype(np.float32)
        ref = reference_outputs(spk_cpu, [xin])[0]
        mine = harness.run_spk(spk_gpu, [xin])[0][0]
        np.testing.assert_allclose(mine, ref, rtol=1e-6, atol=1e-6, err_msg=f"{op} {kh}x{kw} s{sh}x{sw} {pads}")
        checked += 1
