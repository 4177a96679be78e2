"""Pinning the CPU oracle (CPU-only tests).

The restatement (oracle/harness.py + oracle_ops.c) is checked against the
reference runtime built from the reference sources (oracle/_ref) and against
the known-answer vectors of the reference's own C kernel tests; its INT8 core
is checked against exact integer arithmetic and round-half-even ties.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import kat
from conftest import compile_pair, reference_outputs, seeded_input


@pytest.fixture(scope="module")
def oracle(built):
    from oracle import harness

    return harness


@pytest.mark.parametrize("case", sorted(kat.CASES))
def test_reference_runtime_and_oracle_pass_reference_kats(oracle, case):
    from spinnv2_b200.compiler import pipeline

    graph, inputs, expected = kat.CASES[case]()
    spk = pipeline.package(graph, "cpu_ref_large")
    ref = reference_outputs(spk, inputs)
    mine, _ = oracle.run_spk(spk, inputs)
    for r, m, e in zip(ref, mine, expected):
        np.testing.assert_allclose(r, e, rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(m, e, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name,kind", [("lenet5", "uniform"), ("conv3x3_64_56", "normal"),
                                       ("conv7x7s2_3_64_224", "normal"), ("conv3x3s2_128_128_56", "normal"),
                                       ("conv1x1_256_64_56", "normal"), ("gemm_2048_1000", "normal")])
def test_oracle_matches_reference_runtime(oracle, name, kind):
    spk = compile_pair(name, 1, targets=("cuda_b200", "cpu_generic_x86"))
    from spinnv2_b200.spk import read_spk

    x = seeded_input(read_spk(spk["cuda_b200"]).inputs[0].shape, kind)
    ref = reference_outputs(spk["cpu_generic_x86"], [x])
    mine, _ = oracle.run_spk(spk["cuda_b200"], [x])
    for r, m in zip(ref, mine):
        np.testing.assert_allclose(m, r, rtol=1e-5, atol=1e-5)


def test_oracle_matches_reference_runtime_on_yolo_scores(oracle):
    spk = compile_pair("yolo_style", 1)
    x = seeded_input((1, 3, 640, 640), "uniform")
    ref = reference_outputs(spk["cpu_generic_x86"], [x])
    mine, _ = oracle.run_spk(spk["cuda_b200"], [x])
    np.testing.assert_allclose(mine[0], ref[0], rtol=1e-5, atol=1e-5)


def test_round_half_even_known_answers(oracle):
    lib = oracle.oracle_lib()
    cases = [(2.5, -128, 2), (3.5, -128, 4), (-2.5, -128, -2), (-3.5, -128, -4), (0.5, -128, 0), (1.5, -128, 2),
             (127.5, -128, 127), (300.0, -128, 127), (-300.0, -128, -128), (-0.4, 0, 0), (-7.0, 0, 0), (126.5, 0, 126)]
    for v, lo, want in cases:
        assert lib.oracle_sat_rne(ctypes.c_float(v), lo) == want, (v, lo)


def test_int8_conv_accumulators_are_exact(oracle):
    rng = np.random.default_rng(5)
    x = rng.integers(-128, 128, (2, 32, 9, 9), dtype=np.int8)
    w = rng.integers(-128, 128, (16, 32, 3, 3), dtype=np.int8)

    class A:
        strides, pads, dilations, group, fused_activation = [1, 1], [1, 1, 1, 1], [1, 1], 1, 0

    s = oracle.conv_shape(x.shape, w.shape, (2, 16, 9, 9), A)
    acc = np.zeros((2, 16, 9, 9), dtype=np.int32)
    y = np.zeros((2, 16, 9, 9), dtype=np.int8)
    m = np.full(16, 1e-3, dtype=np.float32)
    oracle.oracle_lib().oracle_conv2d_i8(x.ctypes.data, w.ctypes.data, None, m.ctypes.data, None, 0.0,
                                         y.ctypes.data, acc.ctypes.data, ctypes.byref(s))
    xp = np.pad(x.astype(np.int64), ((0, 0), (0, 0), (1, 1), (1, 1)))
    want = np.zeros((2, 16, 9, 9), dtype=np.int64)
    for r in range(3):
        for c in range(3):
            want += np.einsum("nchw,mc->nmhw", xp[:, :, r:r + 9, c:c + 9], w[:, :, r, c].astype(np.int64))
    np.testing.assert_array_equal(acc, want.astype(np.int32))
    expect_q = np.clip(np.rint(want.astype(np.float32) * np.float32(1e-3)), -128, 127).astype(np.int8)
    np.testing.assert_array_equal(y, expect_q)
