"""fp32 numpy forward of a fused graph, for activation-range calibration.

The reference calibrates with onnxruntime's MinMax calibrator
(compiler/quantization/calibrate.py); onnxruntime is not part of this
target's toolchain, so the INT8 flow computes the same statistic, the
max-abs of every activation over a set of seeded inputs, with this plain
numpy forward of the already fused graph (Conv with folded BN, fused
activation and fused residual Add; MaxPool; ReduceMean; Flatten; Gemm;
Softmax; Relu; Add; Sigmoid; Mul).  It runs in float32 with BLAS matmuls, so
its last bits depend on the host; `quantize.py` rounds the ranges up to 11
significant bits before they become scales.
"""

from __future__ import annotations

from typing import Callable

import numpy as np

from .ir import Graph


def _conv(x: np.ndarray, w: np.ndarray, attrs: dict) -> np.ndarray:
    if int(attrs.get("group", 1)) != 1:
        raise NotImplementedError("calibration forward: grouped Conv")
    sh, sw = [int(v) for v in attrs.get("strides", [1, 1])]
    pt, pl, pb, pr = [int(v) for v in attrs.get("pads", [0, 0, 0, 0])]
    dh, dw = [int(v) for v in attrs.get("dilations", [1, 1])]
    m, c, kh, kw = w.shape
    n = x.shape[0]
    xp = np.pad(x, ((0, 0), (0, 0), (pt, pb), (pl, pr)))
    hp, wp = xp.shape[2], xp.shape[3]
    oh = (hp - dh * (kh - 1) - 1) // sh + 1
    ow = (wp - dw * (kw - 1) - 1) // sw + 1
    s = xp.strides
    cols = np.lib.stride_tricks.as_strided(
        xp, shape=(n, oh, ow, c, kh, kw),
        strides=(s[0], s[2] * sh, s[3] * sw, s[1], s[2] * dh, s[3] * dw), writeable=False)
    a = np.ascontiguousarray(cols).reshape(n * oh * ow, c * kh * kw)
    y = a @ w.reshape(m, -1).T
    return np.ascontiguousarray(y.reshape(n, oh, ow, m).transpose(0, 3, 1, 2))


def _maxpool(x: np.ndarray, attrs: dict) -> np.ndarray:
    kh, kw = [int(v) for v in attrs["kernel_shape"]]
    sh, sw = [int(v) for v in attrs.get("strides", [1, 1])]
    pt, pl, pb, pr = [int(v) for v in attrs.get("pads", [0, 0, 0, 0])]
    xp = np.pad(x, ((0, 0), (0, 0), (pt, pb), (pl, pr)), constant_values=-np.inf)
    oh = (xp.shape[2] - kh) // sh + 1
    ow = (xp.shape[3] - kw) // sw + 1
    out = np.full((x.shape[0], x.shape[1], oh, ow), -np.inf, dtype=np.float32)
    for r in range(kh):
        for q in range(kw):
            np.maximum(out, xp[:, :, r:r + sh * (oh - 1) + 1:sh, q:q + sw * (ow - 1) + 1:sw], out=out)
    return out


def _act(y: np.ndarray, act) -> np.ndarray:
    if act in (None, "", "None"):
        return y
    if act == "Relu":
        return np.maximum(y, 0, dtype=np.float32)
    if act == "Silu":
        return (y / (1.0 + np.exp(-y))).astype(np.float32)
    raise NotImplementedError(f"calibration forward: activation {act}")


def _gemm(a: np.ndarray, b: np.ndarray, c, attrs: dict) -> np.ndarray:
    if int(attrs.get("transA", 0)):
        a = a.T
    if int(attrs.get("transB", 0)):
        b = b.T
    y = np.float32(attrs.get("alpha", 1.0)) * (a @ b)
    if c is not None:
        y = y + np.float32(attrs.get("beta", 1.0)) * c
    return y.astype(np.float32)


def forward(graph: Graph, inputs: list[np.ndarray], observe: Callable[[int, np.ndarray], None]) -> None:
    """Run `graph` on `inputs` (batch-major fp32), calling observe(tensor id,
    value) for every graph input and every node output.  Constants come from
    the graph; activations are dropped after their last consumer."""
    last_use: dict[int, int] = {}
    for n in graph.nodes:
        for t in n.inputs:
            last_use[t] = n.id
    env: dict[int, np.ndarray] = {}
    for tid, x in zip(graph.inputs, inputs):
        env[tid] = np.asarray(x, dtype=np.float32)
        observe(tid, env[tid])

    def val(tid: int) -> np.ndarray:
        if tid in env:
            return env[tid]
        return graph.tensors[tid].array().astype(np.float32)

    for n in graph.nodes:
        op, a = n.op_type, n.attrs
        ins = [val(t) for t in n.inputs]
        if op == "Conv":
            y = _conv(ins[0], ins[1], a)
            if len(ins) > 2:
                y += ins[2].reshape(1, -1, 1, 1)
            if len(ins) > 3:
                y += ins[3]
            y = _act(y, a.get("fused_activation"))
        elif op == "MaxPool":
            y = _maxpool(ins[0], a)
        elif op == "ReduceMean":
            axes = tuple(int(v) for v in a.get("axes", [2, 3]))
            y = ins[0].mean(axis=axes, keepdims=bool(int(a.get("keepdims", 1))), dtype=np.float32)
        elif op in ("Flatten", "Reshape"):
            y = ins[0].reshape(ins[0].shape[0], -1) if op == "Flatten" else ins[0].reshape(
                [ins[0].shape[0]] + list(graph.tensors[n.outputs[0]].shape[1:]))
        elif op == "Gemm":
            y = _gemm(ins[0], ins[1], ins[2] if len(ins) > 2 else None, a)
            y = _act(y, a.get("fused_activation"))
        elif op == "Softmax":
            axis = int(a.get("axis", -1))
            e = np.exp(ins[0] - ins[0].max(axis=axis, keepdims=True))
            y = (e / e.sum(axis=axis, keepdims=True)).astype(np.float32)
        elif op == "Relu":
            y = np.maximum(ins[0], 0, dtype=np.float32)
        elif op == "Add":
            y = _act(ins[0] + ins[1], a.get("fused_activation"))
        elif op == "Mul":
            y = ins[0] * ins[1]
        elif op == "Sigmoid":
            y = (1.0 / (1.0 + np.exp(-ins[0]))).astype(np.float32)
        else:
            raise NotImplementedError(f"calibration forward: {op}")
        out = n.outputs[0]
        env[out] = np.asarray(y, dtype=np.float32)
        observe(out, env[out])
        for t in n.inputs:
            if last_use.get(t) == n.id and t in env and t not in graph.outputs:
                del env[t]


def max_abs_ranges(graph: Graph, images: int = 32, seed: int = 1000, chunk: int = 8) -> dict[int, float]:
    """max |x| of every activation over `images` seeded N(0,1) inputs."""
    shape = list(graph.tensors[graph.inputs[0]].shape[1:])
    rng = np.random.default_rng(seed)
    data = rng.standard_normal([images] + shape, dtype=np.float32)
    ranges: dict[int, float] = {}

    def observe(tid: int, v: np.ndarray) -> None:
        m = float(np.max(np.abs(v))) if v.size else 0.0
        ranges[tid] = max(ranges.get(tid, 0.0), m)

    for s in range(0, images, chunk):
        forward(graph, [data[s:s + chunk]], observe)
    return ranges


__all__ = ["forward", "max_abs_ranges"]
