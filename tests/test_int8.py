"""INT8 path: the compiler's quantiser (pinned against the reference weight
quantiser), the oracle's int8 network, and on the GPU the tcgen05 kind::i8
kernels bit-exact against the oracle in int32 accumulators and in the
requantised int8 outputs.

Requantisation contract (same in the oracle and on the GPU):
  a = acc + b_q[c]; v = fp32(a) * M[c]; v += fp32(r) * R; y = clamp(rne(v), lo, 127)
with M[c] = fp32(s_x * s_w[c]) / s_y, R = s_r / s_y, every operation rounded
to nearest in fp32.
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import zlib

import numpy as np
import pytest

from conftest import REPO, compile_pair, seeded_input

GOLDEN = json.loads((REPO / "tests" / "golden" / "spk_sha256.json").read_text())


# ---------------------------------------------------------------- compiler


def test_weight_quantiser_matches_reference_golden():
    """quantize_weights_per_channel over every Conv weight of the fused
    ResNet-50 equals the reference quantize_conv_weights output (W_q bytes
    and scales), recorded by tests/golden/make_golden.py."""
    from spinnv2_b200.compiler import builders
    from spinnv2_b200.compiler.passes import run_pass_pipeline
    from spinnv2_b200.compiler.profile import load_target_profile
    from spinnv2_b200.compiler.quantize import quantize_weights_per_channel

    g = builders.build_config("resnet50", 1)
    run_pass_pipeline(g, profile=load_target_profile("cpu_generic_x86"))
    h = hashlib.sha256()
    count = 0
    for n in g.nodes:
        if n.op_type != "Conv" or int(n.attrs.get("group", 1)) != 1:
            continue
        w_q, s = quantize_weights_per_channel(g.tensors[n.inputs[1]].array())
        h.update(w_q.tobytes())
        h.update(np.asarray(s.tolist(), dtype=np.float64).tobytes())
        count += 1
    want = GOLDEN["resnet50_weight_quant"]
    assert count == want["tensors"]
    assert h.hexdigest() == want["sha256"]


def test_range_rounding_and_bias_quantisation():
    from spinnv2_b200.compiler.quantize import quantize_bias, round_range_up

    for v in (1e-9, 0.3, 1.0, 3.1415926, 127.0, 5.5e4):
        r = round_range_up(v)
        assert r >= np.float32(v) or v < 1e-8
        m, _ = np.frexp(r)
        assert float(m * 2048) == int(m * 2048)  # at most 11 significant bits
        assert r <= v * (1 + 2.0 ** -10) + 1e-8
    assert round_range_up(1.0) == 1.0
    b = np.array([0.5, -0.5, 1.5, 2.5e-3, -7.0], dtype=np.float32)
    sw = np.array([1.0, 1.0, 1.0, 1e-3, 0.5], dtype=np.float32)
    q = quantize_bias(b, 1.0, sw)
    assert q.dtype == np.int32
    np.testing.assert_array_equal(q, [0, 0, 2, 2, -14])  # half to even: 0.5 -> 0, 1.5 -> 2, 2.5 -> 2


@pytest.fixture(scope="module")
def r50_int8():
    from spinnv2_b200.compiler import pipeline

    return pipeline.compile_config("resnet50", 2, targets=("cuda_b200",), int8=True)["cuda_b200"]


def test_quantised_resnet50_structure(r50_int8):
    from spinnv2_b200.spk import read_spk

    pkg = read_spk(r50_int8)
    convs = [n for n in pkg.nodes if n.op_type == "Conv"]
    stem = convs[0]
    assert pkg.tensors[stem.inputs[0]].np_dtype == np.float32
    assert pkg.tensors[stem.inputs[1]].np_dtype == np.float32
    assert pkg.tensors[stem.outputs[0]].np_dtype == np.int8
    for n in convs[1:]:
        assert pkg.tensors[n.inputs[0]].np_dtype == np.int8
        assert pkg.tensors[n.inputs[1]].np_dtype == np.int8
        assert pkg.tensors[n.inputs[2]].np_dtype == np.int32
        assert pkg.tensors[n.outputs[0]].np_dtype == np.int8
        assert len(pkg.quant[n.inputs[1]].scales) == pkg.tensors[n.inputs[1]].shape[0]
        assert pkg.specs[n.kernel_spec_id].kind == "tc_int8"
    mp = next(n for n in pkg.nodes if n.op_type == "MaxPool")
    assert pkg.quant[mp.inputs[0]].scales[0] == pkg.quant[mp.outputs[0]].scales[0]
    rm = next(n for n in pkg.nodes if n.op_type == "ReduceMean")
    assert pkg.tensors[rm.inputs[0]].np_dtype == np.int8 and pkg.tensors[rm.outputs[0]].np_dtype == np.float32
    gemm = next(n for n in pkg.nodes if n.op_type == "Gemm")
    assert pkg.tensors[gemm.inputs[1]].np_dtype == np.float32


def test_int8_network_in_the_oracle_tracks_fp32(r50_int8):
    """Sanity of the quantisation itself: the oracle's INT8 ResNet-50 keeps
    the fp32 network's top-1 and its logits within 5 % of the fp32 scale."""
    from oracle import harness
    from spinnv2_b200.spk import read_spk

    x = seeded_input((2, 3, 224, 224))
    _, env8 = harness.run_spk(r50_int8, [x], keep_all=True)
    spkf = compile_pair("resnet50", 2)
    _, envf = harness.run_spk(spkf["cuda_b200"], [x], keep_all=True)
    g8 = next(n for n in read_spk(r50_int8).nodes if n.op_type == "Gemm")
    gf = next(n for n in read_spk(spkf["cuda_b200"]).nodes if n.op_type == "Gemm")
    l8, lf = env8[g8.outputs[0]], envf[gf.outputs[0]]
    assert np.abs(l8 - lf).max() < 0.05 * np.abs(lf).max()
    np.testing.assert_array_equal(np.argmax(l8, 1), np.argmax(lf, 1))


# ---------------------------------------------------------------- single int8 convs

CASES = {
    # name: (N, C, H, M, k, stride, pad, residual, act)
    "3x3s1_64_res_relu": (2, 64, 20, 64, 3, 1, 1, True, "Relu"),
    "3x3s2_128_256_relu": (3, 128, 15, 256, 3, 2, 1, False, "Relu"),
    "1x1_256_1024_res": (4, 256, 7, 1024, 1, 1, 0, True, "Relu"),
    "1x1_48_40_noact": (2, 48, 9, 40, 1, 1, 0, False, None),
    "1x1s2_64_128": (2, 64, 14, 128, 1, 2, 0, False, "Relu"),
    "7x7s2_16_32": (1, 16, 23, 32, 7, 2, 3, False, "Relu"),
    "3x3s1_256_res": (2, 256, 14, 256, 3, 1, 1, True, "Relu"),
    "5x5s1p2_128_96": (2, 128, 11, 96, 5, 1, 2, False, None),
}


def _int8_conv_graph(case: str, out_i32: bool = False):
    """input(int8) -> MaxPool 1x1 (an internal NHWC int8 copy) -> Conv
    [+ residual MaxPool of a second input] -> output.  Returns (graph, quant
    params, inputs)."""
    from spinnv2_b200.compiler.ir import DTYPE_INT8, DTYPE_INT32, GraphBuilder
    from spinnv2_b200.compiler.quantize import QuantParam

    n, c, h, m, k, s, p, res, act = CASES[case]
    rng = np.random.default_rng(zlib.crc32(case.encode()))
    oh = (h + 2 * p - k) // s + 1
    b = GraphBuilder(f"i8_{case}")
    pool = {"kernel_shape": [1, 1], "strides": [1, 1], "pads": [0, 0, 0, 0]}
    x0 = b.input("x", [n, c, h, h], DTYPE_INT8)
    x = b.op("MaxPool", [x0], [n, c, h, h], pool, out_dtype=DTYPE_INT8)
    w = b.weight("w", rng.integers(-128, 128, (m, c, k, k), dtype=np.int8), DTYPE_INT8)
    bias = b.weight("b", rng.integers(-3000, 3000, m, dtype=np.int32), DTYPE_INT32)
    ins = [x, w, bias]
    inputs = [rng.integers(-128, 128, (n, c, h, h), dtype=np.int8)]
    if res and not out_i32:
        r0 = b.input("r", [n, m, oh, oh], DTYPE_INT8)
        ins.append(b.op("MaxPool", [r0], [n, m, oh, oh], pool, out_dtype=DTYPE_INT8))
        inputs.append(rng.integers(-128, 128, (n, m, oh, oh), dtype=np.int8))
    attrs = {"kernel_shape": [k, k], "strides": [s, s], "pads": [p] * 4, "dilations": [1, 1], "group": 1}
    if act and not out_i32:
        attrs["fused_activation"] = act
    y = b.op("Conv", ins, [n, m, oh, oh], attrs, out_dtype=DTYPE_INT32 if out_i32 else DTYPE_INT8)
    out = y
    if not out_i32:  # keep the conv output internal (NHWC), as inside a network
        out = b.op("MaxPool", [y], [n, m, oh, oh], pool, out_dtype=DTYPE_INT8)
    b.mark_output(out)
    g = b.graph
    sx = 0.05
    q = [QuantParam(x0, "per_tensor", 0, 1, [sx], [0]), QuantParam(x, "per_tensor", 0, 1, [sx], [0]),
         QuantParam(w, "per_channel", 0, m, (rng.random(m) * 4e-3 + 1e-4).astype(np.float32).tolist(), [0] * m)]
    if not out_i32:
        sy = float(np.float32(2.0 + rng.random()))
        q += [QuantParam(y, "per_tensor", 0, 1, [sy], [0]), QuantParam(out, "per_tensor", 0, 1, [sy], [0])]
    if len(ins) > 3:
        q += [QuantParam(g.inputs[1], "per_tensor", 0, 1, [0.03], [0]), QuantParam(ins[3], "per_tensor", 0, 1, [0.03], [0])]
    return g, q, inputs


def _package(case: str, out_i32: bool = False):
    from spinnv2_b200.compiler import pipeline

    g, q, inputs = _int8_conv_graph(case, out_i32)
    return pipeline.package(g, "cuda_b200", quant_params=q), inputs


def _oracle_acc(spk: bytes, inputs) -> np.ndarray:
    """int32 accumulators + b_q of the package's conv, from the oracle."""
    from oracle import harness
    from spinnv2_b200.spk import read_spk

    pkg = read_spk(spk)
    conv = next(n for n in pkg.nodes if n.op_type == "Conv")
    x = inputs[0]
    w = np.ascontiguousarray(pkg.weight(conv.inputs[1]))
    bq = np.ascontiguousarray(pkg.weight(conv.inputs[2]))
    yt = pkg.tensors[conv.outputs[0]]
    s = harness.conv_shape(x.shape, w.shape, yt.shape, conv.attr)
    acc = np.empty(yt.shape, dtype=np.int32)
    y8 = np.empty(yt.shape, dtype=np.int8)
    ones = np.ones(w.shape[0], dtype=np.float32)
    harness.oracle_lib().oracle_conv2d_i8(x.ctypes.data, w.ctypes.data, None, ones.ctypes.data, None, 0.0,
                                          y8.ctypes.data, acc.ctypes.data, ctypes.byref(s))
    return acc + bq.reshape(1, -1, 1, 1)


def test_int8_conv_graphs_run_in_the_oracle():
    """The single-conv cases exercise the requantisation (outputs neither
    constant nor all saturated) and their accumulators stay far from int32
    overflow."""
    from oracle import harness

    for case in CASES:
        spk, inputs = _package(case)
        out = harness.run_spk(spk, inputs)[0][0]
        assert out.dtype == np.int8 and out.std() > 1.0, case
        assert (np.abs(out.astype(np.int32)) == 127).mean() < 0.5, case
        spk32, inputs32 = _package(case, out_i32=True)
        acc = _oracle_acc(spk32, inputs32)
        assert acc.dtype == np.int32 and np.abs(acc).max() < 2**30, case


@pytest.mark.gpu
@pytest.mark.parametrize("case", list(CASES))
def test_int8_conv_bit_exact(gpu, case):
    from oracle import harness
    from spinnv2_b200.runtime import Runtime

    spk, inputs = _package(case)
    ref = harness.run_spk(spk, inputs)[0][0]
    with Runtime(spk, device=0) as rt:
        out = rt.run(*inputs)[0]
        variant = rt.node_variant(next(n.id for n in rt.package.nodes if n.op_type == "Conv"))
    k, s, c, m = CASES[case][4], CASES[case][5], CASES[case][1], CASES[case][3]
    assert variant.startswith("tc_int8") and (("tmastore" in variant) == (m % 16 == 0)), variant
    if k == 1 and s == 1:
        assert "_tma" in variant, variant
    elif c % 128 == 0:
        assert "_im2col" in variant, variant
    np.testing.assert_array_equal(out, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["3x3s1_64_res_relu", "1x1_256_1024_res", "1x1_48_40_noact", "7x7s2_16_32",
                                  "3x3s2_128_256_relu", "5x5s1p2_128_96"])
def test_int8_conv_int32_accumulators_bit_exact(gpu, case):
    from spinnv2_b200.runtime import Runtime

    spk, inputs = _package(case, out_i32=True)
    with Runtime(spk, device=0) as rt:
        out = rt.run(*inputs)[0]
        variant = rt.node_variant(next(n.id for n in rt.package.nodes if n.op_type == "Conv"))
    assert variant.startswith("tc_int8") and variant.endswith("_i32out"), variant
    np.testing.assert_array_equal(out, _oracle_acc(spk, inputs))


@pytest.mark.gpu
def test_int8_resnet50_bs2_every_node_against_the_oracle(gpu, r50_int8):
    """Run INT8 ResNet-50 on the GPU, then re-run every node in the oracle on
    the GPU's own inputs to that node: int8 conv / MaxPool outputs and the
    int8 ReduceMean are bit-exact; the fp32-math stem conv (int8 output) may
    differ by one code where fp32 summation order moves a value across a
    rounding boundary; the fp32 head is within the fp32 tolerance."""
    from oracle import harness
    from spinnv2_b200.runtime import Runtime
    from spinnv2_b200.spk import read_spk

    pkg = read_spk(r50_int8)
    x = seeded_input((2, 3, 224, 224))
    with Runtime(r50_int8, device=0) as rt:
        probs = rt.run(x)[0]
        # The memory plan reuses buffers (the graph input's too, after its
        # last reader), so stage the input again and read each node's
        # outputs right after that node runs.
        rt.set_input(0, x)
        gpu = {}
        for n in pkg.nodes:
            rt.run_nodes(n.id, n.id + 1)
            for t in n.outputs:
                gpu[t] = rt.read_tensor(t)
        variants = {n.id: rt.node_variant(n.id) for n in pkg.nodes}
    gpu[pkg.inputs[0].id] = x
    convs = [n for n in pkg.nodes if n.op_type == "Conv"]
    assert all(variants[n.id].startswith("tc_int8") for n in convs[1:]), variants
    stem_checked = False
    for n in pkg.nodes:
        env = {t: gpu[t] for t in n.inputs if t in gpu}
        want = harness.run_node(pkg, n, env)
        got = gpu[n.outputs[0]]
        if n.op_type == "Conv" and n.id == convs[0].id:
            diff = np.abs(got.astype(np.int32) - want[0].astype(np.int32))
            assert diff.max() <= 1 and (diff > 0).mean() < 1e-3, (n.id, diff.max(), (diff > 0).mean())
            stem_checked = True
        elif got.dtype == np.int8 or n.op_type == "ReduceMean":
            np.testing.assert_array_equal(got, want[0], err_msg=f"node {n.id} {n.op_type}")
        else:  # fp32 head: max-abs 1e-3 plus rel 1e-4 of the tensor's scale
            err = float(np.max(np.abs(got - want[0])))
            assert err <= 1e-3 + 1e-4 * float(np.max(np.abs(want[0]))), (n.id, n.op_type, err)
    assert stem_checked
    _, env = harness.run_spk(r50_int8, [x], keep_all=True)
    assert np.array_equal(np.argmax(probs, 1), np.argmax(env[pkg.outputs[0].id], 1))
