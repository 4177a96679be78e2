"""INT8 quantisation of a fused ResNet-style graph for the CUDA target.

Weights follow the reference quantiser (compiler/quantization/
quantize_weights.py:24-83, `quantize_conv_weights`): per output channel,
symmetric, computed in float32:

    s_w[c] = max(max|W[c]|, 1e-8) / 127
    W_q[c] = clip(round_half_even(W[c] / s_w[c]), -128, 127)

Activations are per-tensor symmetric, s = max|x| / 127 with max|x| taken over
seeded N(0,1) calibration inputs (the reference's `build_activation_quant_
params`, :86-120, takes the same statistic from onnxruntime's calibrator).
The ranges are rounded up to 11 significant bits first, so the package bytes
do not depend on the host BLAS's summation order.

The reference runs only the conv itself in int8 and keeps fp32 activations
between layers (runtime kernels/optimized/conv/conv_int8.c).  This target
keeps activations in int8 between convs and requantises in each conv's
epilogue, with this contract (applied identically by the CPU oracle and the
GPU kernels):

    acc  = sum(x_q * w_q) (int32) + b_q[c],  b_q[c] = rne(b[c] / (s_x * s_w[c]))
    v    = fp32(acc) * M[c],                 M[c] = fp32(s_x * s_w[c]) / s_y
    v    = v + fp32(r_q) * R                 (fused residual, R = s_r / s_y)
    y_q  = clamp(rne(v), 0 if Relu else -128, 127)

with every multiply and add rounded to nearest in fp32 (no fused
multiply-add).  The first conv (graph input in fp32) keeps fp32 weights and
math and quantises its output, y_q = clamp(rne(act(v) * (1 / s_y))); MaxPool
keeps int8 codes and its input's scale; ReduceMean turns int8 back into fp32
(float(sum) * (s_x / denom)); the final Gemm and Softmax stay fp32.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .calibrate import max_abs_ranges
from .ir import DTYPE_FP32, DTYPE_INT8, DTYPE_INT32, Graph

RANGE_BITS = 11  # significant bits kept (rounding up) in calibrated ranges


@dataclass
class QuantParam:
    """One quantisation record (reference quantize_weights.py:14-21)."""

    tensor_id: int
    scheme: str
    quant_axis: int
    num_channels: int
    scales: list[float]
    zero_points: list[int] = field(default_factory=list)


def round_range_up(v: float, bits: int = RANGE_BITS) -> float:
    """Smallest float32 >= v with at most `bits` significant bits."""
    v = max(float(v), 1e-8)
    m, e = np.frexp(v)  # v = m * 2**e, 0.5 <= m < 1
    m = np.ceil(m * (1 << bits)) / (1 << bits)
    return float(np.float32(np.ldexp(m, e)))


def quantize_weights_per_channel(w_fp32: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Reference per-channel weight quantiser, float32 arithmetic."""
    out_channels = w_fp32.shape[0]
    w_flat = np.asarray(w_fp32, dtype=np.float32).reshape(out_channels, -1)
    channel_max = np.maximum(np.max(np.abs(w_flat), axis=1), np.float32(1e-8))
    scales = channel_max / np.float32(127.0)
    w_q = np.empty_like(w_flat, dtype=np.int8)
    for c in range(out_channels):
        w_q[c] = np.clip(np.round(w_flat[c] / scales[c]), -128, 127).astype(np.int8)
    return w_q.reshape(w_fp32.shape), scales.astype(np.float32)


def quantize_bias(b: np.ndarray, s_x: float, s_w: np.ndarray) -> np.ndarray:
    """int32 bias b_q[c] = rne(b[c] / (s_x * s_w[c])), the product in fp32."""
    denom = (np.float32(s_x) * s_w.astype(np.float32)).astype(np.float64)
    q = np.rint(b.astype(np.float64) / denom)
    return np.clip(q, -(2 ** 31), 2 ** 31 - 1).astype(np.int32)


INT8_CONSUMERS = {"Conv", "MaxPool", "ReduceMean"}


def quantize_int8_model(graph: Graph, calib_images: int = 32, seed: int = 1000) -> tuple[Graph, list[QuantParam]]:
    """Quantise a fused fp32 graph in place; returns (graph, quant params)."""
    convs = [n for n in graph.nodes if n.op_type == "Conv"]
    if not convs:
        raise ValueError("no Conv to quantise")
    ranges = max_abs_ranges(graph, images=calib_images, seed=seed)
    consumers: dict[int, list] = {}
    for n in graph.nodes:
        for t in n.inputs:
            consumers.setdefault(t, []).append(n)

    # int8 activations: every conv output, and MaxPool outputs of int8 inputs.
    int8: set[int] = set()
    for n in graph.nodes:
        if n.op_type == "Conv":
            int8.add(n.outputs[0])
        elif n.op_type == "MaxPool" and n.inputs[0] in int8:
            int8.add(n.outputs[0])
    for t in int8:
        if t in graph.outputs:
            raise ValueError(f"int8 graph output {graph.tensors[t].name} is not supported")
        for c in consumers.get(t, []):
            if c.op_type not in INT8_CONSUMERS:
                raise ValueError(f"{c.op_type} cannot consume int8 tensor {graph.tensors[t].name}")
            if c.op_type == "Conv" and c.inputs[0] != t and not (len(c.inputs) > 3 and c.inputs[3] == t):
                raise ValueError("int8 tensor used as a conv weight or bias")

    scales: dict[int, float] = {}
    for n in graph.nodes:  # graph order: a MaxPool sees its input's scale
        for t in n.outputs:
            if t not in int8:
                continue
            if n.op_type == "MaxPool":
                scales[t] = scales[n.inputs[0]]
            else:
                scales[t] = float(np.float32(round_range_up(ranges[t]) / np.float32(127.0)))

    params: list[QuantParam] = []
    for t in sorted(int8):
        graph.tensors[t].dtype = DTYPE_INT8
        params.append(QuantParam(t, "per_tensor", 0, 1, [scales[t]], [0]))

    for n in convs:
        x = n.inputs[0]
        if x not in int8:
            continue  # fp32-input conv (the stem): fp32 weights, int8 output
        if n.attrs.get("fused_activation") not in (None, "", "None", "Relu"):
            raise ValueError(f"conv {n.id}: activation {n.attrs.get('fused_activation')} has no int8 form")
        if int(n.attrs.get("group", 1)) != 1:
            raise ValueError(f"conv {n.id}: grouped int8 conv is not supported")
        if len(n.inputs) > 3 and n.inputs[3] not in int8:
            raise ValueError(f"conv {n.id}: fp32 residual into an int8 conv")
        wt = graph.tensors[n.inputs[1]]
        w_q, s_w = quantize_weights_per_channel(wt.array())
        wt.data, wt.dtype = w_q.tobytes(), DTYPE_INT8
        params.append(QuantParam(wt.id, "per_channel", 0, int(w_q.shape[0]), s_w.tolist(), [0] * int(w_q.shape[0])))
        if len(n.inputs) > 2:
            bt = graph.tensors[n.inputs[2]]
            if bt.dtype != DTYPE_FP32:
                raise ValueError(f"conv {n.id}: bias dtype {bt.dtype}")
            b_q = quantize_bias(bt.array(), scales[x], s_w)
            bt.data, bt.dtype = b_q.tobytes(), DTYPE_INT32
    graph.metadata = dict(graph.metadata or {})
    graph.metadata["quantization"] = {"scheme": "int8 symmetric, per-channel weights, per-tensor activations",
                                      "calibration": f"max-abs over {calib_images} N(0,1) inputs, seed {seed}",
                                      "range_bits": RANGE_BITS}
    return graph, params


__all__ = ["QuantParam", "quantize_int8_model", "quantize_weights_per_channel", "quantize_bias",
           "round_range_up"]


def quantize_weights_only(graph: Graph, calib_images: int = 32, seed: int = 1000) -> tuple[Graph, list[QuantParam]]:
    """The reference compiler's own INT8 format (reference quantize_weights.py:
    24-120): every group-1 conv weight becomes int8 per output channel (the
    same quantiser as above) and every conv input gets a per-tensor scale;
    activations, biases and residuals stay fp32 and the runtime quantises
    each conv input on the fly.  The scales come from the max-abs calibration
    above (the reference takes them from onnxruntime's calibrator)."""
    ranges = max_abs_ranges(graph, images=calib_images, seed=seed)
    params: list[QuantParam] = []
    done_w: set[int] = set()
    done_x: set[int] = set()
    for n in graph.nodes:
        if n.op_type != "Conv" or len(n.inputs) < 2 or int(n.attrs.get("group", 1)) != 1:
            continue
        wt = graph.tensors[n.inputs[1]]
        if n.inputs[1] not in done_w and wt.dtype == DTYPE_FP32 and wt.data is not None:
            w_q, s_w = quantize_weights_per_channel(wt.array())
            wt.data = w_q.tobytes()
            wt.dtype = DTYPE_INT8
            params.append(QuantParam(wt.id, "per_channel", 0, int(s_w.size), [float(v) for v in s_w],
                                     [0] * int(s_w.size)))
            done_w.add(wt.id)
        x = n.inputs[0]
        if x not in done_x and x in ranges:
            s = float(np.float32(round_range_up(ranges[x]) / np.float32(127.0)))
            params.append(QuantParam(x, "per_tensor", 0, 1, [s], [0]))
            done_x.add(x)
    return graph, params
