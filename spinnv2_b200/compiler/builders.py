"""SIR graph builders for the benchmark configurations.

ONNX and onnxruntime are not available, so the graphs of the five configs are
written directly in SIR, with seeded random weights:

  lenet5(batch)                 C1  LeNet-5, input U[0,1) 1x28x28
  conv_sweep(case, batch)       C2  single Conv + bias + Relu (or one Gemm)
  resnet(depth, batch)          C3  ResNet-101 v1.5 (C4 uses depth 50)
  yolo_style(batch)             C5  YOLOv10n-style detector, pre-NMS top-300

Weights are Kaiming-normal (std sqrt(2 / fan_in)); biases N(0, 0.01);
BatchNorm gamma U(0.5,1.5), beta N(0,0.1), mean N(0,0.1), var U(0.5,1.5).
BatchNorm, Relu, Sigmoid*Mul and residual Add appear as separate nodes, as an
ONNX import would produce them; the pass pipeline folds them into the convs.
Gemm weights are stored [K, N] with transB = 0.
"""

from __future__ import annotations

import numpy as np

from .ir import DTYPE_FP32, Graph, GraphBuilder


class _Init:
    def __init__(self, seed: int) -> None:
        self.rng = np.random.default_rng(seed)

    def kaiming(self, shape, fan_in: int) -> np.ndarray:
        return (self.rng.standard_normal(shape, dtype=np.float32) * np.float32(np.sqrt(2.0 / fan_in))).astype(np.float32)

    def bias(self, n: int) -> np.ndarray:
        return (self.rng.standard_normal(n, dtype=np.float32) * np.float32(0.01)).astype(np.float32)

    def bn(self, c: int, gamma_scale: float = 1.0) -> list[np.ndarray]:
        gamma = (self.rng.uniform(0.5, 1.5, c).astype(np.float32) * np.float32(gamma_scale)).astype(np.float32)
        beta = (self.rng.standard_normal(c, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
        mean = (self.rng.standard_normal(c, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
        var = self.rng.uniform(0.5, 1.5, c).astype(np.float32)
        return [gamma, beta, mean, var]


def _out_hw(h: int, w: int, k: int, s: int, p: int) -> tuple[int, int]:
    return (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1


class _Net:
    """Op-level helpers over a GraphBuilder."""

    def __init__(self, name: str, seed: int) -> None:
        self.b = GraphBuilder(name)
        self.init = _Init(seed)
        self.n = 0

    def _name(self, kind: str) -> str:
        self.n += 1
        return f"{kind}{self.n}"

    def conv(self, x: int, cout: int, k: int, s: int = 1, p: int | None = None, bias: bool = False,
             bn: bool = False, act: str | None = None, bn_gamma_scale: float = 1.0) -> int:
        nm = self._name("conv")
        n, c, h, w = self.b.shape(x)
        p = k // 2 if p is None else p
        oh, ow = _out_hw(h, w, k, s, p)
        ins = [x, self.b.weight(f"{nm}_w", self.init.kaiming((cout, c, k, k), c * k * k))]
        if bias:
            ins.append(self.b.weight(f"{nm}_b", self.init.bias(cout)))
        y = self.b.op("Conv", ins, [n, cout, oh, ow], {"kernel_shape": [k, k], "strides": [s, s],
                                                       "pads": [p, p, p, p], "dilations": [1, 1], "group": 1},
                      name=nm)
        if bn:
            params = [self.b.weight(f"{nm}_bn{i}", v) for i, v in enumerate(self.init.bn(cout, bn_gamma_scale))]
            y = self.b.op("BatchNormalization", [y] + params, [n, cout, oh, ow], {"epsilon": 1e-5}, name=f"{nm}_bn")
        if act == "Relu":
            y = self.relu(y)
        elif act == "Silu":
            sig = self.b.op("Sigmoid", [y], self.b.shape(y), name=f"{nm}_sig")
            y = self.b.op("Mul", [y, sig], self.b.shape(y), name=f"{nm}_silu")
        return y

    def relu(self, x: int) -> int:
        return self.b.op("Relu", [x], self.b.shape(x))

    def maxpool(self, x: int, k: int, s: int, p: int) -> int:
        n, c, h, w = self.b.shape(x)
        oh, ow = _out_hw(h, w, k, s, p)
        return self.b.op("MaxPool", [x], [n, c, oh, ow], {"kernel_shape": [k, k], "strides": [s, s],
                                                          "pads": [p, p, p, p]})

    def add(self, a: int, c: int) -> int:
        return self.b.op("Add", [a, c], self.b.shape(a))

    def gemm(self, x: int, nout: int) -> int:
        m, k = self.b.shape(x)
        w = self.b.weight(self._name("fc_w"), self.init.kaiming((k, nout), k))
        bias = self.b.weight(self._name("fc_b"), self.init.bias(nout))
        return self.b.op("Gemm", [x, w, bias], [m, nout], {"alpha": 1.0, "beta": 1.0, "transA": 0, "transB": 0})

    def const(self, name: str, values) -> int:
        return self.b.weight(name, np.asarray(values, dtype=np.float32))

    def flatten(self, x: int) -> int:
        s = self.b.shape(x)
        return self.b.op("Flatten", [x], [s[0], int(np.prod(s[1:]))], {"axis": 1})


# ---------------------------------------------------------------- C1

def lenet5(batch: int = 1, seed: int = 0) -> Graph:
    net = _Net(f"lenet5_b{batch}", seed)
    x = net.b.input("input", [batch, 1, 28, 28])
    y = net.conv(x, 6, 5, p=2, bias=True, act="Relu")
    y = net.maxpool(y, 2, 2, 0)
    y = net.conv(y, 16, 5, p=0, bias=True, act="Relu")
    y = net.maxpool(y, 2, 2, 0)
    y = net.flatten(y)
    y = net.relu(net.gemm(y, 120))
    y = net.relu(net.gemm(y, 84))
    y = net.gemm(y, 10)
    net.b.mark_output(y)
    return net.b.graph


# ---------------------------------------------------------------- C2

SWEEP_CASES = {
    # name: (cin, cout, k, stride, pad, hw)  or ("gemm", k, n)
    "conv7x7s2_3_64_224": (3, 64, 7, 2, 3, 224),
    "conv3x3_64_56": (64, 64, 3, 1, 1, 56),
    "conv3x3_128_28": (128, 128, 3, 1, 1, 28),
    "conv3x3_256_14": (256, 256, 3, 1, 1, 14),
    "conv3x3_512_7": (512, 512, 3, 1, 1, 7),
    "conv1x1_256_64_56": (256, 64, 1, 1, 0, 56),
    "conv1x1_1024_256_14": (1024, 256, 1, 1, 0, 14),
    "conv1x1_2048_512_7": (2048, 512, 1, 1, 0, 7),
    "conv3x3s2_128_128_56": (128, 128, 3, 2, 1, 56),
    "gemm_2048_1000": ("gemm", 2048, 1000),
}


def sweep_flops(case: str, batch: int) -> float:
    spec = SWEEP_CASES[case]
    if spec[0] == "gemm":
        return 2.0 * batch * spec[1] * spec[2]
    cin, cout, k, s, p, hw = spec
    oh, ow = _out_hw(hw, hw, k, s, p)
    return 2.0 * batch * cout * oh * ow * cin * k * k


def conv_sweep(case: str, batch: int = 1, seed: int = 0) -> Graph:
    spec = SWEEP_CASES[case]
    net = _Net(f"sweep_{case}_b{batch}", seed)
    if spec[0] == "gemm":
        x = net.b.input("input", [batch, spec[1]])
        y = net.gemm(x, spec[2])
    else:
        cin, cout, k, s, p, hw = spec
        x = net.b.input("input", [batch, cin, hw, hw])
        y = net.conv(x, cout, k, s=s, p=p, bias=True, act="Relu")
    net.b.mark_output(y)
    return net.b.graph


# ---------------------------------------------------------------- C3 / C4

RESNET_LAYERS = {50: [3, 4, 6, 3], 101: [3, 4, 23, 3]}

# Scale of the BatchNorm gamma (drawn from U(0.5, 1.5) like every other BN)
# of the last conv of each residual branch, the BN that feeds the residual
# Add.  With random running statistics the folded BN does not normalise, so
# at gain 1 every bottleneck adds a branch as large as its input and the
# activations grow ~1.8x per block: ResNet-101's logits reach ~1e8-1e9 and
# an fp32 comparison of them measures cancellation, not arithmetic.  A small
# gamma on the branch's last BN (the "zero-init residual" practice of
# training recipes, here 0.2 instead of 0) keeps the logits O(1-100).
RESIDUAL_BN_GAMMA = 0.2


def resnet(depth: int = 101, batch: int = 1, seed: int = 0) -> Graph:
    """ResNet v1.5 (stride on the 3x3), head ReduceMean -> Gemm -> Softmax.
    The BN closing each residual branch has gamma scaled by RESIDUAL_BN_GAMMA."""
    net = _Net(f"resnet{depth}_b{batch}", seed)
    x = net.b.input("input", [batch, 3, 224, 224])
    y = net.conv(x, 64, 7, s=2, p=3, bn=True, act="Relu")
    y = net.maxpool(y, 3, 2, 1)
    cin = 64
    for stage, (blocks, width) in enumerate(zip(RESNET_LAYERS[depth], [64, 128, 256, 512])):
        for i in range(blocks):
            stride = 2 if (i == 0 and stage > 0) else 1
            shortcut = y
            t = net.conv(y, width, 1, bn=True, act="Relu")
            t = net.conv(t, width, 3, s=stride, p=1, bn=True, act="Relu")
            t = net.conv(t, width * 4, 1, bn=True, bn_gamma_scale=RESIDUAL_BN_GAMMA)
            if i == 0:
                shortcut = net.conv(y, width * 4, 1, s=stride, p=0, bn=True)
            y = net.relu(net.add(t, shortcut))
            cin = width * 4
    n = net.b.shape(y)[0]
    y = net.b.op("ReduceMean", [y], [n, cin, 1, 1], {"axes": [2, 3], "keepdims": 1})
    y = net.flatten(y)
    y = net.gemm(y, 1000)
    y = net.b.op("Softmax", [y], net.b.shape(y), {"axis": 1})
    net.b.mark_output(y)
    return net.b.graph


def resnet_gflop_per_image(depth: int) -> float:
    """Algorithmic conv + FC GFLOP per 224x224 image (2 * MACs)."""
    g = resnet(depth, 1)
    flops = 0.0
    for node in g.nodes:
        if node.op_type == "Conv":
            w = g.tensors[node.inputs[1]].shape
            y = g.tensors[node.outputs[0]].shape
            flops += 2.0 * y[1] * y[2] * y[3] * w[1] * w[2] * w[3]
        elif node.op_type == "Gemm":
            w = g.tensors[node.inputs[1]].shape
            flops += 2.0 * w[0] * w[1]
    return flops / 1e9


# ---------------------------------------------------------------- C5

def yolo_style(batch: int = 1, seed: int = 0, size: int = 640, classes: int = 80, topk: int = 300) -> Graph:
    net = _Net(f"yolo_style_b{batch}", seed)
    b = net.b

    def cbs(x, cout, k, s=1):
        return net.conv(x, cout, k, s=s, p=k // 2, bn=True, act="Silu")

    def c2f(x, cout, n, shortcut):
        c = cout // 2
        y = cbs(x, 2 * c, 1)
        nb, _, h, w = b.shape(y)
        parts = b.node("Split", [y], [[nb, c, h, w], [nb, c, h, w]], {"axis": 1})
        outs = list(parts)
        cur = parts[1]
        for _ in range(n):
            t = cbs(cbs(cur, c, 3), c, 3)
            cur = net.add(cur, t) if shortcut else t
            outs.append(cur)
        cat = b.op("Concat", outs, [nb, c * len(outs), h, w], {"axis": 1})
        return cbs(cat, cout, 1)

    def resize2x(x):
        n, c, h, w = b.shape(x)
        return b.op("Resize", [x], [n, c, 2 * h, 2 * w], {"mode": "nearest"})

    def concat(xs):
        n, _, h, w = b.shape(xs[0])
        return b.op("Concat", xs, [n, sum(b.shape(t)[1] for t in xs), h, w], {"axis": 1})

    x = b.input("images", [batch, 3, size, size])
    y = cbs(x, 16, 3, 2)
    y = cbs(y, 32, 3, 2)
    y = c2f(y, 32, 1, True)
    y = cbs(y, 64, 3, 2)
    p3 = c2f(y, 64, 2, True)
    y = cbs(p3, 128, 3, 2)
    p4 = c2f(y, 128, 2, True)
    y = cbs(p4, 256, 3, 2)
    y = c2f(y, 256, 1, True)
    # SPPF
    t = cbs(y, 128, 1)
    m1 = net.maxpool(t, 5, 1, 2)
    m2 = net.maxpool(m1, 5, 1, 2)
    m3 = net.maxpool(m2, 5, 1, 2)
    p5 = cbs(concat([t, m1, m2, m3]), 256, 1)
    # PAN neck
    n4 = c2f(concat([resize2x(p5), p4]), 128, 1, False)
    n3 = c2f(concat([resize2x(n4), p3]), 64, 1, False)
    n4b = c2f(concat([cbs(n3, 64, 3, 2), n4]), 128, 1, False)
    n5b = c2f(concat([cbs(n4b, 128, 3, 2), p5]), 256, 1, False)
    # decoupled heads
    boxes, scores = [], []
    for feat in (n3, n4b, n5b):
        nb, _, h, w = b.shape(feat)
        bx = net.conv(cbs(cbs(feat, 64, 3), 64, 3), 4, 1, p=0, bias=True)
        cl = net.conv(cbs(cbs(feat, 80, 3), 80, 3), classes, 1, p=0, bias=True)
        boxes.append(b.op("Reshape", [bx, net.const(net._name("shape"), [nb, 4, h * w])], [nb, 4, h * w]))
        scores.append(b.op("Reshape", [cl, net.const(net._name("shape"), [nb, classes, h * w])],
                           [nb, classes, h * w]))
    anchors = sum(b.shape(t)[2] for t in boxes)
    box = b.op("Concat", boxes, [batch, 4, anchors], {"axis": 2})
    cls = b.op("Concat", scores, [batch, classes, anchors], {"axis": 2})
    cls = b.op("Sigmoid", [cls], b.shape(cls))
    best = b.op("ReduceMax", [cls], [batch, anchors], {"axes": [1], "keepdims": 0})
    vals, idx = b.node("TopK", [best, net.const("k", [topk])], [[batch, topk], [batch, topk]],
                       {"axis": 1, "largest": 1, "sorted": 1})
    box_t = b.op("Transpose", [box], [batch, anchors, 4], {"perm": [0, 2, 1]})
    idx3 = b.op("Unsqueeze", [idx], [batch, topk, 1], {"axes": [2]})
    idx4 = b.op("Tile", [idx3, net.const("repeats", [1, 1, 4])], [batch, topk, 4])
    sel = b.op("GatherElements", [box_t, idx4], [batch, topk, 4], {"axis": 1})
    b.mark_output(vals)
    b.mark_output(sel)
    return b.graph


# ---------------------------------------------------------------- op coverage

# Single-op graphs for the runtime ops outside the five configs (reference
# compiler/ir/types.py:15-47 op set).  Each is  x -> Add(c) -> OP -> Add(c')
# -> y  so that the op reads and writes arena activations (NHWC on the device
# where rank 4) rather than only the row-major graph IO; cases with a second
# runtime input (an index tensor) take it as a graph input.
OP_CASES = (
    "matmul", "matmul_bcast", "clip", "leakyrelu", "avgpool", "globalavgpool", "mod", "sub", "div",
    "transpose", "tile", "slice_axis1", "slice_axis3", "gather_const", "gather_input", "unsqueeze",
    "topk_ties", "topk_smallest", "topk_long", "softmax_channels", "maxpool_s1_k3", "maxpool_s1_k5",
    "maxpool_s1_k7", "resize_3x2", "resize_frac", "transpose_last2",
)


def op_case(case: str, batch: int = 2, seed: int = 0) -> Graph:
    net = _Net(f"op_{case}_b{batch}", seed)
    b = net.b
    rng = net.init.rng

    def pre(shape):
        x = b.input("input", shape)
        return b.op("Add", [x, net.const("pre_c", [0.125])], shape)

    def post(y):
        y = b.op("Add", [y, net.const("post_c", [-0.25])], b.shape(y))
        b.mark_output(y)
        return b.graph

    n = batch
    if case == "matmul":
        x = pre([n, 3, 40, 24])
        w = b.weight("mm_b", rng.standard_normal((24, 36), dtype=np.float32))
        return post(b.op("MatMul", [x, w], [n, 3, 40, 36]))
    if case == "matmul_bcast":
        x = pre([n, 1, 33, 20])
        w = b.weight("mm_b", rng.standard_normal((3, 20, 70), dtype=np.float32))
        return post(b.op("MatMul", [x, w], [n, 3, 33, 70]))
    if case == "clip":
        x = pre([n, 8, 13, 11])
        return post(b.op("Clip", [x, net.const("lo", [-0.5]), net.const("hi", [0.7])], [n, 8, 13, 11]))
    if case == "leakyrelu":
        x = pre([n, 8, 13, 11])
        return post(b.op("LeakyRelu", [x], [n, 8, 13, 11], {"alpha": 0.1}))
    if case == "avgpool":
        x = pre([n, 8, 15, 15])
        return post(b.op("AveragePool", [x], [n, 8, 8, 8], {"kernel_shape": [3, 3], "strides": [2, 2],
                                                             "pads": [1, 1, 1, 1]}))
    if case.startswith("maxpool_s1_k"):
        # Stride-1 square windows (the SPPF form) with the window's padding.
        # The 5x5 case is wide enough that the GPU kernel walks bands of
        # several output rows, and its prime height leaves a short last band.
        k = int(case[-1])
        shape = {3: [n, 12, 11, 9], 5: [n, 256, 37, 80], 7: [n, 8, 13, 10]}[k]
        x = pre(shape)
        return post(b.op("MaxPool", [x], list(shape), {"kernel_shape": [k, k], "strides": [1, 1],
                                                      "pads": [k // 2] * 4}))
    if case in ("resize_3x2", "resize_frac"):
        # Nearest upsampling by integer factors 3 (H) and 2 (W), and by the
        # non-integer factors 9/6 and 11/7.
        out = [n, 8, 15, 14] if case == "resize_3x2" else [n, 8, 9, 11]
        x = pre([n, 8, 5, 7] if case == "resize_3x2" else [n, 8, 6, 7])
        return post(b.op("Resize", [x], out, {"mode": "nearest"}))
    if case == "globalavgpool":
        x = pre([n, 16, 7, 9])
        return post(b.op("GlobalAveragePool", [x], [n, 16, 1, 1]))
    if case == "mod":
        x = b.input("input", [n, 8, 6, 5])
        y = b.op("Mul", [x, net.const("scale", [7.0])], [n, 8, 6, 5])
        return post(b.op("Mod", [y, net.const("m", [3.0])], [n, 8, 6, 5]))
    if case == "sub":
        x = pre([n, 8, 6, 5])
        c = b.weight("sub_c", rng.standard_normal((8, 1, 1), dtype=np.float32))
        return post(b.op("Sub", [x, c], [n, 8, 6, 5]))
    if case == "div":
        x = pre([n, 8, 6, 5])
        c = b.weight("div_c", rng.uniform(0.5, 2.0, (1, 1, 5)).astype(np.float32))
        return post(b.op("Div", [x, c], [n, 8, 6, 5]))
    if case == "transpose":
        x = pre([n, 8, 5, 6])
        return post(b.op("Transpose", [x], [n, 5, 6, 8], {"perm": [0, 2, 3, 1]}))
    if case == "transpose_last2":
        # The form of the detector head's box transpose ([N, 4, anchors] ->
        # [N, anchors, 4]): the two inner dims swapped, odd sizes on both.
        x = pre([n, 5, 333])
        return post(b.op("Transpose", [x], [n, 333, 5], {"perm": [0, 2, 1]}))
    if case == "tile":
        x = pre([n, 3, 4, 5])
        return post(b.op("Tile", [x, net.const("reps", [1, 2, 1, 3])], [n, 6, 4, 15]))
    if case == "slice_axis1":
        x = pre([n, 16, 10, 12])
        ins = [x, net.const("starts", [3]), net.const("ends", [14]), net.const("axes", [1]), net.const("steps", [2])]
        return post(b.op("Slice", ins, [n, 6, 10, 12]))
    if case == "slice_axis3":
        x = pre([n, 16, 10, 12])
        ins = [x, net.const("starts", [-8]), net.const("ends", [100]), net.const("axes", [-1]),
               net.const("steps", [3])]
        return post(b.op("Slice", ins, [n, 16, 10, 3]))
    if case == "gather_const":
        x = pre([n, 10, 6, 7])
        idx = net.const("idx", np.array([[1, 9], [-1, 0], [4, 4]], dtype=np.float32))
        return post(b.op("Gather", [x, idx], [n, 3, 2, 6, 7], {"axis": 1}))
    if case == "gather_input":
        x = pre([n, 10, 6, 7])
        idx = b.input("indices", [4])
        return post(b.op("Gather", [x, idx], [n, 10, 6, 4], {"axis": 3}))
    if case == "topk_ties":
        # Integer-valued scores (Mod of a scaled input): many equal values,
        # so the order among ties (smaller index first) is exercised.
        x = b.input("input", [n, 4, 500])
        y = b.op("Mul", [x, net.const("scale", [7.0])], [n, 4, 500])
        y = b.op("Mod", [y, net.const("m", [3.0])], [n, 4, 500])
        vals, idx = b.node("TopK", [y, net.const("k", [37])], [[n, 4, 37], [n, 4, 37]], {"axis": -1, "largest": 1})
        b.mark_output(vals)
        b.mark_output(idx)
        return b.graph
    if case == "topk_smallest":
        x = pre([n, 3, 1000])
        vals, idx = b.node("TopK", [x, net.const("k", [100])], [[n, 3, 100], [n, 3, 100]], {"axis": 2, "largest": 0})
        b.mark_output(vals)
        b.mark_output(idx)
        return b.graph
    if case == "softmax_channels":
        # Softmax over the channels of a rank-4 activation (stored channels-
        # last on the device) into a row-major graph output.
        x = pre([n, 21, 12, 10])
        y = b.op("Softmax", [x], [n, 21, 12, 10], {"axis": 1})
        b.mark_output(y)
        return b.graph
    if case == "topk_long":
        # A row longer than the shared-memory sort (40000 scores).
        x = pre([n, 40000])
        vals, idx = b.node("TopK", [x, net.const("k", [50])], [[n, 50], [n, 50]], {"axis": 1, "largest": 1})
        b.mark_output(vals)
        b.mark_output(idx)
        return b.graph
    if case == "unsqueeze":
        x = pre([n, 8, 6])
        return post(b.op("Unsqueeze", [x], [n, 8, 1, 6], {"axes": [2]}))
    raise KeyError(case)


# Protection plan over the FUSED LeNet-5 graph (node ids after the pass
# pipeline: 0 Conv+Relu, 2 Conv+Relu, 5 Gemm, 9 Gemm): range guards on the
# first conv (a Relu output, so [0, 60]) and on the first Gemm (infinite
# bounds: only non-finite values trip it), DMR on the second conv and on
# the logits.  Entries: (node_id, mode, lower, upper).
LENET5_PROTECTION = ((0, "range_guard_rerun", 0.0, 60.0), (2, "dmr_compare_rerun", None, None),
                     (5, "range_guard_rerun", None, None), (9, "dmr_compare_rerun", None, None))


def lenet5_protection_entries(graph: Graph) -> list[dict]:
    """LENET5_PROTECTION as plan entries for the fused LeNet-5 `graph`."""
    out = []
    for nid, mode, lo, hi in LENET5_PROTECTION:
        e = {"node_id": nid, "tensor_id": graph.nodes[nid].outputs[0], "mode": mode}
        if lo is not None:
            e["lower_bound"], e["upper_bound"] = lo, hi
        out.append(e)
    return out


def build_config(name: str, batch: int, seed: int = 0) -> Graph:
    if name.startswith("op_") and name[3:] in OP_CASES:
        return op_case(name[3:], batch, seed)
    if name == "lenet5":
        return lenet5(batch, seed)
    if name == "resnet101":
        return resnet(101, batch, seed)
    if name == "resnet50":
        return resnet(50, batch, seed)
    if name == "yolo_style":
        return yolo_style(batch, seed)
    if name in SWEEP_CASES:
        return conv_sweep(name, batch, seed)
    raise KeyError(name)


__all__ = ["lenet5", "conv_sweep", "resnet", "yolo_style", "op_case", "build_config", "SWEEP_CASES", "OP_CASES",
           "LENET5_PROTECTION", "lenet5_protection_entries",
           "sweep_flops",
           "resnet_gflop_per_image", "DTYPE_FP32"]
