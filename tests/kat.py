"""Known-answer cases taken from the reference runtime's C kernel tests, as
single-op SIR graphs.  Each case returns (graph, inputs, expected outputs).

  relu       runtime/tests/test_kernel_relu.c:10-40
  add        runtime/tests/test_kernel_add.c:8-45 (and broadcast :47-90)
  softmax    runtime/tests/test_kernel_softmax.c:11-50 (properties)
  maxpool    runtime/tests/test_kernel_maxpool.c:15-90 (2x2 s2 on 4x4)
  transpose  runtime/tests/test_kernel_transpose.c:15-55 (perm 0,2,3,1)
"""

from __future__ import annotations

import numpy as np

from spinnv2_b200.compiler.ir import GraphBuilder


def _single(op: str, inputs: list[np.ndarray], out_shape, attrs=None, weights=()) -> tuple:
    b = GraphBuilder(f"kat_{op.lower()}")
    ids = [b.input(f"x{i}", list(x.shape)) for i, x in enumerate(inputs)]
    ids += [b.weight(f"w{i}", w) for i, w in enumerate(weights)]
    y = b.op(op, ids, list(out_shape), attrs or {})
    b.mark_output(y)
    return b.graph


def relu_case():
    x = np.array([-3.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0, 100.0], dtype=np.float32).reshape(1, 1, 1, 8)
    return _single("Relu", [x], x.shape), [x], [np.maximum(x, 0)]


def add_case():
    a = np.arange(16, dtype=np.float32).reshape(1, 4, 2, 2)
    b = (np.arange(16, dtype=np.float32) * 10).reshape(1, 4, 2, 2)
    return _single("Add", [a, b], a.shape), [a, b], [a + b]


def add_broadcast_case():
    a = np.arange(16, dtype=np.float32).reshape(1, 4, 2, 2)
    b = np.array([100, 200, 300, 400], dtype=np.float32).reshape(1, 4, 1, 1)
    return _single("Add", [a, b], a.shape), [a, b], [a + b]


def softmax_case():
    x = np.array([[1.0, 2.0, 3.0, 4.0]], dtype=np.float32)
    e = np.exp(x - x.max())
    return _single("Softmax", [x], x.shape, {"axis": -1}), [x], [e / e.sum()]


def softmax_large_case():
    x = np.array([[1000.0, 1001.0, 1002.0, 1003.0]], dtype=np.float32)
    e = np.exp(x - x.max())
    return _single("Softmax", [x], x.shape, {"axis": -1}), [x], [e / e.sum()]


def maxpool_case():
    x = np.arange(1, 17, dtype=np.float32).reshape(1, 1, 4, 4)
    attrs = {"kernel_shape": [2, 2], "strides": [2, 2], "pads": [0, 0, 0, 0]}
    return _single("MaxPool", [x], (1, 1, 2, 2), attrs), [x], [np.array([6, 8, 14, 16], np.float32).reshape(1, 1, 2, 2)]


def maxpool_negative_case():
    x = np.array([-5, -3, -1, -7, -2, -4, -6, -8, -9, -1, -3, -5, -7, -2, -4, -6], dtype=np.float32).reshape(1, 1, 4, 4)
    attrs = {"kernel_shape": [2, 2], "strides": [2, 2], "pads": [0, 0, 0, 0]}
    return _single("MaxPool", [x], (1, 1, 2, 2), attrs), [x], [np.array([-2, -1, -1, -3], np.float32).reshape(1, 1, 2, 2)]


def transpose_case():
    x = np.arange(24, dtype=np.float32).reshape(1, 2, 3, 4)
    return _single("Transpose", [x], (1, 3, 4, 2), {"perm": [0, 2, 3, 1]}), [x], [np.transpose(x, (0, 2, 3, 1))]


def transpose_middle_case():
    x = np.arange(120, dtype=np.float32).reshape(2, 3, 4, 5)
    return _single("Transpose", [x], (2, 4, 3, 5), {"perm": [0, 2, 1, 3]}), [x], [np.transpose(x, (0, 2, 1, 3))]


CASES = {
    "relu": relu_case, "add": add_case, "add_broadcast": add_broadcast_case, "softmax": softmax_case,
    "softmax_large": softmax_large_case, "maxpool": maxpool_case, "maxpool_negative": maxpool_negative_case,
    "transpose": transpose_case, "transpose_middle": transpose_middle_case,
}
