"""GPU parity: the CUDA runtime (through the C-ABI, spkv2_* entry points)
against the reference SPINNV2 CPU runtime (oracle/_ref, built from the
reference sources) on the same fused graph and the same seeded inputs.

fp32 tolerance: max-abs 1e-3 and rel 1e-4 on final outputs, element-wise,
i.e. np.testing.assert_allclose(gpu, ref, atol=1e-3, rtol=1e-4).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import compile_pair, reference_outputs, seeded_input

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4


def _run_gpu(spk: bytes, inputs, **kw):
    from spinnv2_b200.runtime import Runtime

    with Runtime(spk, device=0, **kw) as rt:
        outs = rt.run(*inputs)
        variants = {rt.package.nodes[i].op_type + ":" + rt.node_variant(i) for i in range(len(rt.package.nodes))}
    return outs, variants


@pytest.mark.parametrize("math", ["spec", "fp32"])
def test_lenet5_matches_reference(gpu, math):
    from spinnv2_b200.runtime import MATH_FP32, MATH_SPEC

    spk = compile_pair("lenet5", 1)
    x = seeded_input((1, 1, 28, 28), "uniform")
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out, variants = _run_gpu(spk["cuda_b200"], [x], math_mode=MATH_FP32 if math == "fp32" else MATH_SPEC)
    np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)


SWEEP = ["conv7x7s2_3_64_224", "conv3x3_64_56", "conv3x3_128_28", "conv3x3_256_14", "conv3x3_512_7",
         "conv1x1_256_64_56", "conv1x1_1024_256_14", "conv1x1_2048_512_7", "conv3x3s2_128_128_56", "gemm_2048_1000"]


@pytest.mark.parametrize("case", SWEEP)
@pytest.mark.parametrize("batch", [1, 4])
def test_sweep_matches_reference(gpu, case, batch):
    spk = compile_pair(case, batch)
    from spinnv2_b200.spk import read_spk

    shape = read_spk(spk["cuda_b200"]).inputs[0].shape
    x = seeded_input(shape)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out, _ = _run_gpu(spk["cuda_b200"], [x])
    np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)


def test_resnet101_bs1_matches_reference(gpu):
    """Softmax outputs and the pre-softmax logits (an extra graph output of
    the same fused graph, so the reference runtime computes them too),
    element-wise."""
    from conftest import compile_with_outputs, gemm_output

    spk = compile_with_outputs("resnet101", 1, gemm_output)
    x = seeded_input((1, 3, 224, 224))
    ref_probs, ref_logits = reference_outputs(spk["cpu_generic_x86"], [x])
    (probs, logits), _ = _run_gpu(spk["cuda_b200"], [x])
    print("3xtf32 resnet101 bs1 logits max abs err", float(np.max(np.abs(logits - ref_logits))),
          "max |logit|", float(np.max(np.abs(ref_logits))))
    np.testing.assert_allclose(logits, ref_logits, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(probs, ref_probs, atol=ATOL, rtol=RTOL)


def test_resnet101_bs2_graph_replay_is_stable(gpu):
    from spinnv2_b200.runtime import Runtime

    spk = compile_pair("resnet101", 2)
    x = seeded_input((2, 3, 224, 224), seed=7)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    with Runtime(spk["cuda_b200"], device=0, graph=True) as rt:
        runs = [rt.run(x)[0] for _ in range(4)]  # eager, capture, replay, replay
    for r in runs:
        np.testing.assert_allclose(r, ref, atol=ATOL, rtol=RTOL)
    for r in runs[1:]:
        np.testing.assert_array_equal(r, runs[0])


@pytest.mark.parametrize("rows", [16, 64, 100])
def test_gemm_rows_on_tensor_cores_match_reference(gpu, rows):
    spk = compile_pair("gemm_2048_1000", rows)
    x = seeded_input((rows, 2048))
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out, variants = _run_gpu(spk["cuda_b200"], [x])
    assert any("gemm_as_tc_3xtf32" in v for v in variants), variants
    np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("case", ["conv7x7s2_3_64_224", "conv1x1_256_64_56", "conv3x3_512_7", "conv3x3s2_128_128_56"])
def test_sweep_batch32_matches_reference(gpu, case):
    from spinnv2_b200.spk import read_spk

    spk = compile_pair(case, 32)
    x = seeded_input(read_spk(spk["cuda_b200"]).inputs[0].shape)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out, _ = _run_gpu(spk["cuda_b200"], [x])
    np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)


def test_resnet101_tf32_mode_is_close(gpu):
    """Plain TF32 is the fast mode, not the parity mode: the tensor core reads
    each fp32 operand as TF32 (low 13 mantissa bits dropped, weights rounded
    to nearest when packed), about 2^-10 relative per activation.  Over
    ResNet-101's 104 convolutions (logits up to ~70) that must keep the top-1
    class, stay within 2 % of the logit scale and within 1e-2 absolute on the
    softmax outputs (measured on B200: 0.47 % and 4.6e-3)."""
    from conftest import compile_with_outputs, gemm_output
    from spinnv2_b200.runtime import MATH_TF32

    spk = compile_with_outputs("resnet101", 2, gemm_output)
    x = seeded_input((2, 3, 224, 224), seed=11)
    ref_probs, ref_logits = reference_outputs(spk["cpu_generic_x86"], [x])
    (probs, logits), _ = _run_gpu(spk["cuda_b200"], [x], math_mode=MATH_TF32)
    err = float(np.max(np.abs(probs - ref_probs)))
    rel = float(np.max(np.abs(logits - ref_logits)) / np.max(np.abs(ref_logits)))
    print("tf32 resnet101 softmax max abs", err, "logits max rel", rel)
    assert err < 1e-2
    assert rel < 2e-2
    np.testing.assert_array_equal(np.argmax(probs, axis=1), np.argmax(ref_probs, axis=1))


@pytest.mark.parametrize("case", ["conv3x3_256_14", "conv1x1_1024_256_14"])
@pytest.mark.parametrize("math", ["3xtf32", "tf32"])
def test_sweep_batch32_on_cta_pairs_matches_reference(gpu, case, math, monkeypatch):
    """2-SM tiles (opt-in): one M = 256 MMA per CTA pair, each CTA holding
    half of the weight panel, same numerics as single tiles."""
    from spinnv2_b200.runtime import MATH_3XTF32, MATH_TF32
    from spinnv2_b200.spk import read_spk

    monkeypatch.setenv("SPKV2_TC_PAIR", "1")
    spk = compile_pair(case, 32)
    x = seeded_input(read_spk(spk["cuda_b200"]).inputs[0].shape)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out, variants = _run_gpu(spk["cuda_b200"], [x], math_mode=MATH_3XTF32 if math == "3xtf32" else MATH_TF32)
    assert any("_pair_" in v for v in variants), variants
    if math == "3xtf32":
        np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)
    else:
        assert float(np.max(np.abs(out[0] - ref))) < 2e-2 * float(np.max(np.abs(ref)))


def _tail_tolerance(out, ref, math):
    if math == "3xtf32":
        np.testing.assert_allclose(out, ref, atol=ATOL, rtol=RTOL)
    else:
        assert float(np.max(np.abs(out - ref))) < 2e-2 * float(np.max(np.abs(ref)))


@pytest.mark.parametrize("case", ["conv3x3_256_14", "conv1x1_1024_256_14"])
@pytest.mark.parametrize("math", ["3xtf32"])
def test_stream_k_tail_matches_reference_and_repeats_bit_exact(gpu, case, math):
    """Batch 32 leaves fewer tiles than SMs, so the tiles' K steps are spread
    evenly over all CTAs (two to four segments per tile; 3xTF32 math, the
    mode that uses stream-K).  The partials are
    added in segment order by whichever epilogue warp arrives last, so a
    second context reproduces the output bit for bit."""
    from spinnv2_b200.runtime import MATH_3XTF32, MATH_TF32
    from spinnv2_b200.spk import read_spk

    mode = MATH_3XTF32 if math == "3xtf32" else MATH_TF32
    spk = compile_pair(case, 32)
    x = seeded_input(read_spk(spk["cuda_b200"]).inputs[0].shape)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out, variants = _run_gpu(spk["cuda_b200"], [x], math_mode=mode)
    assert any("_sk_" in v for v in variants), variants
    _tail_tolerance(out[0], ref, math)
    again, _ = _run_gpu(spk["cuda_b200"], [x], math_mode=mode)
    np.testing.assert_array_equal(out[0], again[0])


def test_stream_k_off_agrees_with_stream_k(gpu, monkeypatch):
    """SPKV2_TC_NO_STREAMK=1 keeps whole tiles per CTA: same result up to the
    order of the fp32 adds."""
    from spinnv2_b200.spk import read_spk

    spk = compile_pair("conv3x3_512_7", 32)
    x = seeded_input(read_spk(spk["cuda_b200"]).inputs[0].shape)
    on, v_on = _run_gpu(spk["cuda_b200"], [x])
    monkeypatch.setenv("SPKV2_TC_NO_STREAMK", "1")
    off, v_off = _run_gpu(spk["cuda_b200"], [x])
    split = ("_sk_", "_splitk_")
    assert any(k in v for v in v_on for k in split) and not any(k in v for v in v_off for k in split), (v_on, v_off)
    np.testing.assert_allclose(on[0], off[0], atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("math", ["3xtf32"])
def test_stream_k_with_residual_and_relu_matches_reference(gpu, math):
    """Residual add + Relu fused into a stream-K conv: the warp that finishes
    a split tile loads the residual tile and applies the activation."""
    import copy

    from spinnv2_b200.compiler import builders, pipeline
    from spinnv2_b200.runtime import MATH_3XTF32, MATH_TF32

    net = builders._Net("sk_residual", 3)
    x_id = net.b.input("input", [32, 256, 14, 14])
    y = net.conv(x_id, 256, 3, s=1, p=1, bias=True)
    net.b.mark_output(net.relu(net.add(y, x_id)))
    graph = pipeline.fuse(net.b.graph)
    spk_gpu = pipeline.package(copy.deepcopy(graph), "cuda_b200")
    spk_cpu = pipeline.package(copy.deepcopy(graph), "cpu_generic_x86")
    x = seeded_input((32, 256, 14, 14), seed=5)
    ref = reference_outputs(spk_cpu, [x])[0]
    out, variants = _run_gpu(spk_gpu, [x], math_mode=MATH_3XTF32 if math == "3xtf32" else MATH_TF32)
    assert any("_sk_" in v for v in variants), variants
    _tail_tolerance(out[0], ref, math)


@pytest.mark.parametrize("case,batch", [("conv3x3_512_7", 32), ("conv3x3_256_14", 1), ("conv1x1_2048_512_7", 1),
                                        ("conv3x3_128_28", 1), ("gemm_2048_1000", 16)])
@pytest.mark.parametrize("math", ["3xtf32", "tf32"])
def test_split_k_over_all_tiles_matches_reference_and_repeats_bit_exact(gpu, case, batch, math):
    """Few tiles (at most half the SMs): every CTA takes an even share of all
    tiles' K steps and parks its partial sums; the reduce kernel adds each
    tile's segments in CTA order and applies bias and activation.  The
    order is fixed, so a second context reproduces the output bit for bit."""
    from spinnv2_b200.runtime import MATH_3XTF32, MATH_TF32
    from spinnv2_b200.spk import read_spk

    mode = MATH_3XTF32 if math == "3xtf32" else MATH_TF32
    spk = compile_pair(case, batch)
    x = seeded_input(read_spk(spk["cuda_b200"]).inputs[0].shape, seed=13)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])[0]
    out, variants = _run_gpu(spk["cuda_b200"], [x], math_mode=mode)
    assert any("_splitk_" in v for v in variants), variants
    _tail_tolerance(out[0], ref, math)
    again, _ = _run_gpu(spk["cuda_b200"], [x], math_mode=mode)
    np.testing.assert_array_equal(out[0], again[0])


def test_split_k_with_residual_and_relu_matches_reference(gpu):
    """Residual add + Relu fused into a split-K conv at batch 1: the reduce
    kernel adds bias, then the residual, then applies the activation."""
    import copy

    from spinnv2_b200.compiler import builders, pipeline

    net = builders._Net("splitk_residual", 3)
    x_id = net.b.input("input", [1, 256, 14, 14])
    y = net.conv(x_id, 256, 3, s=1, p=1, bias=True)
    net.b.mark_output(net.relu(net.add(y, x_id)))
    graph = pipeline.fuse(net.b.graph)
    spk_gpu = pipeline.package(copy.deepcopy(graph), "cuda_b200")
    spk_cpu = pipeline.package(copy.deepcopy(graph), "cpu_generic_x86")
    x = seeded_input((1, 256, 14, 14), seed=6)
    ref = reference_outputs(spk_cpu, [x])[0]
    out, variants = _run_gpu(spk_gpu, [x])
    assert any("_splitk_" in v for v in variants), variants
    np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("cout,k", [(4, 1), (10, 3), (17, 3)])
@pytest.mark.parametrize("batch", [2, 64])
def test_narrow_output_convs_on_tensor_cores_match_reference(gpu, cout, k, batch):
    """Convs with fewer than 32 output channels (the detector's 4-channel box
    head) run in one 32-column tensor-core tile with direct stores."""
    import copy

    from spinnv2_b200.compiler import builders, pipeline

    net = builders._Net(f"narrow_{cout}_{k}", 7)
    x_id = net.b.input("input", [batch, 64, 20, 20])
    net.b.mark_output(net.conv(x_id, cout, k, s=1, p=k // 2, bias=True, act="Relu" if k == 3 else None))
    graph = pipeline.fuse(net.b.graph)
    spk_gpu = pipeline.package(copy.deepcopy(graph), "cuda_b200")
    spk_cpu = pipeline.package(copy.deepcopy(graph), "cpu_generic_x86")
    x = seeded_input((batch, 64, 20, 20), seed=8)
    ref = reference_outputs(spk_cpu, [x])[0]
    out, variants = _run_gpu(spk_gpu, [x])
    assert any(v.startswith("Conv:tc_3xtf32") for v in variants), variants
    np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("cin,k,pad,hw,cout,batch", [
    (3, 7, 3, (224, 224), 64, 2),  # ResNet stem
    (3, 7, 3, (31, 29), 64, 3),    # odd extents: the last s2d row / column is half padding
    (3, 3, 1, (64, 64), 16, 2),    # detector stem
    (3, 3, 1, (33, 17), 32, 1),
    (1, 5, 2, (28, 28), 20, 2),    # even padding: taps start at the sub-pixel 0
    (4, 4, 1, (20, 22), 64, 2),    # even kernel
    (2, 3, 0, (15, 15), 40, 2),    # no padding
])
@pytest.mark.parametrize("math", ["spec", "tf32"])
def test_stride2_few_channel_convs_space_to_depth_match_reference(gpu, cin, k, pad, hw, cout, batch, math):
    """Stride-2 convs over <= 4 channels (a network's first conv) run as a
    stride-1 conv over the 2 x 2 space-to-depth input (16 channels, two-tap
    im2col TMA): against the reference, and in TF32 mode against the row-packed
    / re-laid-out path (SPKV2_TC_NO_S2D) on the same package."""
    import copy
    import os

    from spinnv2_b200.compiler import builders, pipeline
    from spinnv2_b200.runtime import MATH_SPEC, MATH_TF32

    net = builders._Net(f"s2d_{cin}_{k}_{pad}", 9)
    shape = [batch, cin, hw[0], hw[1]]
    x_id = net.b.input("input", shape)
    net.b.mark_output(net.conv(x_id, cout, k, s=2, p=pad, bias=True, act="Relu"))
    graph = pipeline.fuse(net.b.graph)
    spk_gpu = pipeline.package(copy.deepcopy(graph), "cuda_b200")
    x = seeded_input(tuple(shape), seed=12)
    mode = MATH_TF32 if math == "tf32" else MATH_SPEC
    out, variants = _run_gpu(spk_gpu, [x], math_mode=mode)
    assert any("_s2d" in v and "_im2col2tap" in v for v in variants), variants
    if math == "spec":
        spk_cpu = pipeline.package(copy.deepcopy(graph), "cpu_generic_x86")
        ref = reference_outputs(spk_cpu, [x])[0]
        np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)
    else:
        os.environ["SPKV2_TC_NO_S2D"] = "1"
        try:
            base, base_variants = _run_gpu(spk_gpu, [x], math_mode=mode)
        finally:
            del os.environ["SPKV2_TC_NO_S2D"]
        assert not any("_s2d" in v for v in base_variants), base_variants
        # Same TF32 products, different summation order.
        np.testing.assert_allclose(out[0], base[0], atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("cin,cout,k,stride,hw,amode", [
    (16, 16, 3, 1, (40, 36), "_im2col2tap"),   # C % 16 == 0: two 16-channel im2col columns per K step
    (16, 32, 3, 2, (41, 40), "_im2col2tap"),
    (16, 64, 1, 1, (20, 20), "_im2col2tap"),
    (80, 80, 3, 1, (20, 18), "_im2col2tap"),   # C % 32 == 16: K steps cross filter taps
    (48, 32, 3, 2, (21, 22), "_im2col2tap"),
    (48, 32, 1, 1, (40, 40), "_tma"),          # 1x1, C % 32 != 0: the last K step reads zeros past C
    (80, 80, 1, 1, (20, 22), "_tma"),
])
@pytest.mark.parametrize("math", ["spec", "tf32"])
def test_tma_fed_convs_with_channel_counts_off_32_match_reference(gpu, cin, cout, k, stride, hw, amode, math):
    import copy

    from spinnv2_b200.compiler import builders, pipeline
    from spinnv2_b200.runtime import MATH_SPEC, MATH_TF32

    net = builders._Net(f"c{cin}_{cout}_{k}_{stride}", 10)
    shape = [2, cin, hw[0], hw[1]]
    x_id = net.b.input("input", shape)
    y = net.conv(x_id, cin, 1, s=1, p=0, bias=True)  # the tested conv reads an NHWC device tensor
    net.b.mark_output(net.conv(y, cout, k, s=stride, p=k // 2, bias=True, act="Relu"))
    graph = pipeline.fuse(net.b.graph)
    spk_gpu = pipeline.package(copy.deepcopy(graph), "cuda_b200")
    spk_cpu = pipeline.package(copy.deepcopy(graph), "cpu_generic_x86")
    x = seeded_input(tuple(shape), seed=13)
    ref = reference_outputs(spk_cpu, [x])[0]
    from spinnv2_b200.runtime import Runtime

    with Runtime(spk_gpu, device=0, math_mode=MATH_TF32 if math == "tf32" else MATH_SPEC) as rt:
        out = rt.run(x)
        convs = [n.id for n in rt.package.nodes if n.op_type == "Conv"]
        tested = rt.node_variant(convs[-1])
    assert amode + "_" in tested, tested  # the conv under test reads its A operand in that mode
    if math == "spec":
        np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)
    else:
        np.testing.assert_allclose(out[0], ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("widths", [(8, 12, 4), (6, 10), (16, 16, 16, 16)])
def test_split_and_concat_match_reference(gpu, widths):
    """Channel Split and Concat between convs (NHWC on the device): 16-byte
    row segments take the row-copy kernel, odd channel counts the generic
    strided one; results are copies, so they must match exactly."""
    import copy

    from spinnv2_b200.compiler import builders, pipeline

    net = builders._Net("split_concat", 4)
    b = net.b
    total = sum(widths)
    x = b.input("input", [3, 8, 9, 11])
    y = net.conv(x, total, 1, s=1, p=0, bias=True)
    parts = list(b.node("Split", [y], [[3, w, 9, 11] for w in widths], {"axis": 1}))
    parts = [net.conv(t, w, 3, s=1, p=1, bias=True, act="Relu") for t, w in zip(parts, widths)]
    cat = b.op("Concat", parts[::-1], [3, total, 9, 11], {"axis": 1})
    b.mark_output(net.conv(cat, 5, 1, s=1, p=0, bias=True))
    graph = pipeline.fuse(net.b.graph)
    spk_gpu = pipeline.package(copy.deepcopy(graph), "cuda_b200")
    spk_cpu = pipeline.package(copy.deepcopy(graph), "cpu_generic_x86")
    xin = seeded_input((3, 8, 9, 11), seed=9)
    ref = reference_outputs(spk_cpu, [xin])[0]
    out, variants = _run_gpu(spk_gpu, [xin])
    kinds = {v for v in variants if v.startswith(("Split:", "Concat:"))}
    assert len(kinds) == 2, variants
    np.testing.assert_allclose(out[0], ref, atol=ATOL, rtol=RTOL)
