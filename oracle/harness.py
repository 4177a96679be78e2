"""CPU interpreter of SPK packages - TEST INFRASTRUCTURE ONLY.

Executes an SPK node by node on the host in logical NCHW order: Conv through
the C restatement (oracle_ops.c: reference scalar conv loop for fp32, the
INT8 requantisation contract for int8), everything else in numpy following
the reference kernels' semantics (runtime/kernels/reference/*):
  MaxPool maxpool.c:5-43, Resize resize.c:5-31, Concat concat.c, Split split.c,
  Add add.c (+fused act), Mul/Sub/Div binary.c, Sigmoid sigmoid.c, Softmax
  softmax.c, ReduceMean/Max reduce.c, TopK topk.c (descending, ties to the
  smaller index, fp32 indices), GatherElements gather_elements.c, Transpose
  transpose.c, Tile tile.c, Gemm gemm.c (alpha, per-column bias, beta
  ignored), Flatten/Reshape/Unsqueeze/Cast copy in logical order.
INT8 extras (no reference counterpart): int8 MaxPool keeps codes; int8
ReduceMean returns (float)sum(codes) * (s_x / denom).
Returns every tensor, so tests can check single nodes.
"""

from __future__ import annotations

import ctypes

import numpy as np

from spinnv2_b200.spk import SpkPackage, read_spk

from . import ORACLE_LIB


class _ConvShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in
                ("N", "C", "H", "W", "M", "KH", "KW", "OH", "OW", "sh", "sw", "ph", "pw", "dh", "dw", "group", "act")]


_olib = None


def oracle_lib() -> ctypes.CDLL:
    global _olib
    if _olib is None:
        if not ORACLE_LIB.exists():
            raise FileNotFoundError(f"{ORACLE_LIB} missing: build it with `make -C oracle oracle`")
        lib = ctypes.CDLL(str(ORACLE_LIB))
        vp = ctypes.c_void_p
        lib.oracle_conv2d_f32.argtypes = [vp, vp, vp, vp, vp, ctypes.POINTER(_ConvShape)]
        lib.oracle_conv2d_f32_to_i8.argtypes = [vp, vp, vp, vp, ctypes.POINTER(_ConvShape), ctypes.c_float]
        lib.oracle_conv2d_i8.argtypes = [vp, vp, vp, vp, vp, ctypes.c_float, vp, vp, ctypes.POINTER(_ConvShape)]
        lib.oracle_dequant_w8.argtypes = [vp, vp, vp, vp, vp, ctypes.POINTER(_ConvShape)]
        lib.oracle_sat_rne.argtypes = [ctypes.c_float, ctypes.c_int]
        lib.oracle_sat_rne.restype = ctypes.c_int
        _olib = lib
    return _olib


def _ptr(a):
    return None if a is None else a.ctypes.data


def conv_shape(x_shape, w_shape, y_shape, attr) -> _ConvShape:
    s = _ConvShape()
    s.N, s.C, s.H, s.W = x_shape
    s.M, _, s.KH, s.KW = w_shape
    s.OH, s.OW = y_shape[2], y_shape[3]
    s.sh, s.sw = attr.strides
    s.ph, s.pw = attr.pads[0], attr.pads[1]
    s.dh, s.dw = (attr.dilations[0] or 1), (attr.dilations[1] or 1)
    s.group = attr.group if attr.group > 0 else 1
    s.act = attr.fused_activation
    return s


def requant_scales(pkg: SpkPackage, node) -> tuple[np.ndarray, float]:
    """M[c] = fp32(s_x * s_w[c]) / s_y and R = s_r / s_y, in fp32."""
    sx = np.float32(pkg.quant[node.inputs[0]].scales[0])
    sy = np.float32(pkg.quant[node.outputs[0]].scales[0])
    sw = pkg.quant[node.inputs[1]].scales.astype(np.float32)
    m = ((sx * sw).astype(np.float32) / sy).astype(np.float32)
    r = np.float32(0.0)
    if len(node.inputs) > 3:
        r = np.float32(np.float32(pkg.quant[node.inputs[3]].scales[0]) / sy)
    return m, float(r)


def run_conv(pkg: SpkPackage, node, env: dict, acc_out: np.ndarray | None = None) -> np.ndarray:
    lib = oracle_lib()
    x = np.ascontiguousarray(env[node.inputs[0]])
    w = np.ascontiguousarray(pkg.weight(node.inputs[1]))
    yt = pkg.tensors[node.outputs[0]]
    s = conv_shape(x.shape, w.shape, yt.shape, node.attr)
    b = np.ascontiguousarray(pkg.weight(node.inputs[2])) if len(node.inputs) > 2 else None
    res = np.ascontiguousarray(env[node.inputs[3]]) if len(node.inputs) > 3 else None
    y = np.empty(yt.shape, dtype=yt.np_dtype)
    if x.dtype == np.float32 and w.dtype == np.int8 and y.dtype == np.float32:
        # Weights-only INT8 (the reference compiler's format, reference
        # kernels/optimized/conv/conv_int8.c:22-56,86-119): x quantised per
        # tensor, q = sat8(rne(x * fp32(1 / s_x))) (the reference's vector
        # lanes; its scalar tail uses round-half-away and only runs for
        # images whose C*H*W is not a multiple of 16), int8 conv to int32,
        # then the fused dequantise.
        sx = np.float32(pkg.quant[node.inputs[0]].scales[0])
        inv = np.float32(np.float32(1.0) / sx)
        xq = np.ascontiguousarray(np.clip(np.rint((x * inv).astype(np.float32)), -128, 127).astype(np.int8))
        acc = np.empty(yt.shape, dtype=np.int32)
        ones = np.ones(s.M, dtype=np.float32)
        scratch = np.empty(yt.shape, dtype=np.int8)
        lib.oracle_conv2d_i8(_ptr(xq), _ptr(w), None, _ptr(ones), None, 0.0, _ptr(scratch), _ptr(acc),
                             ctypes.byref(s))
        cs = np.ascontiguousarray((pkg.quant[node.inputs[1]].scales.astype(np.float32) * sx).astype(np.float32))
        lib.oracle_dequant_w8(_ptr(acc), _ptr(cs), _ptr(b), _ptr(res), _ptr(y), ctypes.byref(s))
    elif x.dtype == np.float32 and y.dtype == np.float32:
        lib.oracle_conv2d_f32(_ptr(x), _ptr(w), _ptr(b), _ptr(res), _ptr(y), ctypes.byref(s))
    elif x.dtype == np.float32 and y.dtype == np.int8:
        inv = np.float32(1.0) / np.float32(pkg.quant[node.outputs[0]].scales[0])
        lib.oracle_conv2d_f32_to_i8(_ptr(x), _ptr(w), _ptr(b), _ptr(y), ctypes.byref(s), float(inv))
    elif x.dtype == np.int8:
        m, r = requant_scales(pkg, node)
        m = np.ascontiguousarray(m)
        lib.oracle_conv2d_i8(_ptr(x), _ptr(w), _ptr(b), _ptr(m), _ptr(res), r, _ptr(y), _ptr(acc_out),
                             ctypes.byref(s))
    else:
        raise NotImplementedError(f"conv dtypes {x.dtype}->{y.dtype}")
    return y


def _act(v: np.ndarray, act: int) -> np.ndarray:
    if act == 1:
        return np.where(v > 0, v, np.float32(0)).astype(np.float32)
    if act == 2:
        return (v / (np.float32(1) + np.exp(-v))).astype(np.float32)
    return v


def _pool(x, attr, kind):
    n, c, h, w = x.shape
    kh, kw = attr.kernel_shape
    sh, sw = attr.strides
    ph, pw = attr.pads[0], attr.pads[1]
    oh = (h + attr.pads[0] + attr.pads[2] - kh) // sh + 1
    ow = (w + attr.pads[1] + attr.pads[3] - kw) // sw + 1
    if x.dtype == np.int8:
        pad_val = -128
    else:
        pad_val = -np.inf
    xp = np.full((n, c, h + 2 * ph + kh, w + 2 * pw + kw), pad_val, dtype=x.dtype)
    xp[:, :, ph:ph + h, pw:pw + w] = x
    out = None
    for r in range(kh):
        for s in range(kw):
            win = xp[:, :, r:r + sh * oh:sh, s:s + sw * ow:sw][:, :, :oh, :ow]
            out = win.copy() if out is None else np.maximum(out, win)
    return out


def _resize(x, yshape):
    n, c, h, w = x.shape
    oh, ow = yshape[2], yshape[3]
    scale_h = np.float32(oh) / np.float32(h)
    scale_w = np.float32(ow) / np.float32(w)
    ih = np.minimum(np.floor(np.arange(oh, dtype=np.float32) / scale_h).astype(np.int64), h - 1)
    iw = np.minimum(np.floor(np.arange(ow, dtype=np.float32) / scale_w).astype(np.int64), w - 1)
    return x[:, :, ih][:, :, :, iw]


def _axes(pkg, node, rank):
    attr = node.attr
    if len(node.inputs) > 1:
        vals = pkg.weight(node.inputs[1]).reshape(-1)
        return [int(v) % rank for v in vals]
    if attr.extra:
        return [a % rank for a in attr.extra]
    return list(range(rank))


def run_node(pkg: SpkPackage, node, env: dict) -> list[np.ndarray]:
    op = node.op_type
    a = node.attr
    ins = [env[t] if t in env else pkg.weight(t) for t in node.inputs]
    outs = [pkg.tensors[t] for t in node.outputs]
    if op == "Conv":
        return [run_conv(pkg, node, env)]
    if op == "Gemm":
        A = ins[0].T if a.trans_a else ins[0]
        B = ins[1].T if a.trans_b else ins[1]
        y = (np.float32(a.alpha) * (A.astype(np.float32) @ B.astype(np.float32))).astype(np.float32)
        if len(ins) > 2:
            y = (y + ins[2].reshape(-1)[None, :]).astype(np.float32)
        return [y]
    if op == "MaxPool":
        return [_pool(ins[0], a, "max")]
    if op in ("Relu",):
        return [np.where(ins[0] > 0, ins[0], np.float32(0)).astype(np.float32)]
    if op == "Sigmoid":
        return [(np.float32(1) / (np.float32(1) + np.exp(-ins[0]))).astype(np.float32)]
    if op in ("Flatten", "Reshape", "Unsqueeze", "Cast"):
        return [np.ascontiguousarray(ins[0]).reshape(outs[0].shape)]
    if op == "Add":
        return [_act((ins[0] + ins[1]).astype(np.float32), a.fused_activation)]
    if op == "Sub":
        return [(ins[0] - ins[1]).astype(np.float32)]
    if op == "Mul":
        return [(ins[0] * ins[1]).astype(np.float32)]
    if op == "Div":
        return [(ins[0] / ins[1]).astype(np.float32)]
    if op == "Concat":
        return [np.concatenate(ins, axis=a.axis % len(outs[0].shape))]
    if op == "Split":
        axis = a.axis % len(ins[0].shape)
        cuts = np.cumsum([o.shape[axis] for o in outs])[:-1]
        return [np.ascontiguousarray(p) for p in np.split(ins[0], cuts, axis=axis)]
    if op == "Resize":
        return [_resize(ins[0], outs[0].shape)]
    if op in ("ReduceMean", "ReduceMax"):
        x = ins[0]
        axes = tuple(_axes(pkg, node, x.ndim))
        if op == "ReduceMax":
            y = np.max(x, axis=axes, keepdims=bool(a.keepdims))
        elif x.dtype == np.int8:
            denom = np.float32(1)
            for ax in axes:
                denom = np.float32(denom * np.float32(x.shape[ax]))
            factor = np.float32(np.float32(pkg.quant[node.inputs[0]].scales[0]) / denom)
            s = np.sum(x.astype(np.int32), axis=axes, keepdims=bool(a.keepdims)).astype(np.float32)
            y = (s * factor).astype(np.float32)
        else:
            denom = np.float32(1)
            for ax in axes:
                denom = np.float32(denom * np.float32(x.shape[ax]))
            y = np.sum((x / denom).astype(np.float32), axis=axes, keepdims=bool(a.keepdims), dtype=np.float32)
        return [np.ascontiguousarray(y.reshape(outs[0].shape))]
    if op == "Softmax":
        x = ins[0]
        axis = a.axis % x.ndim
        e = np.exp((x - np.max(x, axis=axis, keepdims=True)).astype(np.float32)).astype(np.float32)
        return [(e / np.sum(e, axis=axis, keepdims=True, dtype=np.float32)).astype(np.float32)]
    if op == "TopK":
        x = ins[0]
        axis = a.axis % x.ndim
        k = min(int(ins[1].reshape(-1)[0]), x.shape[axis])
        order = np.argsort(-x if a.largest else x, axis=axis, kind="stable")
        idx = np.take(order, np.arange(k), axis=axis)
        vals = np.take_along_axis(x, idx, axis=axis)
        return [vals.astype(np.float32), idx.astype(np.float32)]
    if op == "GatherElements":
        axis = a.axis % ins[0].ndim
        idx = ins[1].astype(np.int64)
        idx = np.where(idx < 0, idx + ins[0].shape[axis], idx)
        return [np.take_along_axis(ins[0], idx, axis=axis)]
    if op == "Transpose":
        perm = a.extra if a.extra else list(range(ins[0].ndim))
        return [np.ascontiguousarray(np.transpose(ins[0], perm))]
    if op == "Tile":
        reps = [o // i for o, i in zip(outs[0].shape, ins[0].shape)]
        return [np.tile(ins[0], reps)]
    if op == "MatMul":
        # reference/mm/matmul.c:3-50: leading dims broadcast, fp32 sums.
        return [np.matmul(ins[0], ins[1]).astype(np.float32).reshape(outs[0].shape)]
    if op == "Clip":
        # reference/activation/clip_leakyrelu.c:5-29: min/max from inputs 1/2.
        lo = ins[1].reshape(-1)[0] if len(ins) > 1 else np.float32(-np.inf)
        hi = ins[2].reshape(-1)[0] if len(ins) > 2 else np.float32(np.inf)
        v = np.where(ins[0] < lo, lo, ins[0])
        return [np.where(v > hi, hi, v).astype(np.float32)]
    if op == "LeakyRelu":
        # reference/activation/clip_leakyrelu.c:31-50: v >= 0 ? v : v * alpha.
        x = ins[0]
        return [np.where(x >= 0, x, x * np.float32(a.alpha)).astype(np.float32)]
    if op == "AveragePool":
        return [_avgpool(ins[0], a, outs[0].shape)]
    if op == "GlobalAveragePool":
        # reference/pool/avgpool.c:49-71: sum * (1 / (H*W)).
        x = ins[0]
        inv = np.float32(1) / np.float32(x.shape[2] * x.shape[3])
        s = np.sum(x, axis=(2, 3), keepdims=True, dtype=np.float32)
        return [(s * inv).astype(np.float32)]
    if op == "Mod":
        # reference/math/binary.c:25-27: (float)((int)a % (int)b), C remainder
        # (truncating division: the sign follows a).
        av = ins[0].astype(np.int32)
        bv = np.broadcast_to(ins[1].astype(np.int32), np.broadcast_shapes(ins[0].shape, ins[1].shape))
        return [np.fmod(np.broadcast_to(av, bv.shape), bv).astype(np.float32)]
    if op == "Slice":
        return [_slice(ins, node, outs[0].shape)]
    if op == "Gather":
        # reference/tensor/gather.c:4-44: fp32 indices, negative ones wrap.
        axis = a.axis % ins[0].ndim
        idx = ins[1].astype(np.int64)
        idx = np.where(idx < 0, idx + ins[0].shape[axis], idx)
        return [np.take(ins[0], idx, axis=axis).reshape(outs[0].shape)]
    raise NotImplementedError(op)


def _avgpool(x, attr, yshape):
    """reference/pool/avgpool.c:3-47: mean over the in-range taps only
    (padding is not counted), fp32 sums in tap order."""
    n, c, h, w = x.shape
    oh, ow = yshape[2], yshape[3]
    kh, kw = attr.kernel_shape
    sh, sw = attr.strides
    ph, pw = attr.pads[0], attr.pads[1]
    out = np.zeros((n, c, oh, ow), dtype=np.float32)
    for i in range(oh):
        for j in range(ow):
            s = np.zeros((n, c), dtype=np.float32)
            cnt = 0
            for r in range(kh):
                ih = i * sh + r - ph
                if ih < 0 or ih >= h:
                    continue
                for q in range(kw):
                    iw = j * sw + q - pw
                    if iw < 0 or iw >= w:
                        continue
                    s = (s + x[:, :, ih, iw]).astype(np.float32)
                    cnt += 1
            out[:, :, i, j] = s / np.float32(cnt) if cnt else np.float32(0)
    return out


def _slice(ins, node, yshape):
    """reference/tensor/slice.c:4-56: one axis from starts[0], ends[0],
    axes[0] (default 0), steps[0] (default 1); negative start/end wrap,
    end clamps to the axis size, start clamps at 0."""
    x = ins[0]
    start, end = int(ins[1].reshape(-1)[0]), int(ins[2].reshape(-1)[0])
    axis = int(ins[3].reshape(-1)[0]) if len(ins) > 3 else 0
    step = int(ins[4].reshape(-1)[0]) if len(ins) > 4 else 1
    axis %= x.ndim
    dim = x.shape[axis]
    start = start + dim if start < 0 else start
    end = end + dim if end < 0 else end
    end = min(end, dim)
    start = max(start, 0)
    count = max(0, (end - start + step - 1) // step)
    sel = start + step * np.arange(count)
    return np.ascontiguousarray(np.take(x, sel, axis=axis)).reshape(yshape)


def run_spk(spk: bytes | SpkPackage, inputs: list[np.ndarray], keep_all: bool = False):
    """Run a package on the CPU. Returns (outputs, env of every tensor)."""
    pkg = spk if isinstance(spk, SpkPackage) else read_spk(spk)
    env: dict[int, np.ndarray] = {}
    for t, x in zip(pkg.inputs, inputs):
        env[t.id] = np.ascontiguousarray(x, dtype=t.np_dtype).reshape(t.shape)
    for node in pkg.nodes:
        for tid, val in zip(node.outputs, run_node(pkg, node, env)):
            env[tid] = val
    outs = [env[t.id] for t in pkg.outputs]
    return outs, (env if keep_all else None)
