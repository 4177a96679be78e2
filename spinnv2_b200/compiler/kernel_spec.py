"""KernelSpec selection and scratch sizing.

For the CPU profiles the selection rules, kinds and scratch formulas are the
reference planner's (compiler/planner/kernel_spec.py:71-298): ordered profile
tokens pick (backend, kind) per node, a `ref` token adds a fallback spec, the
scratch arena is the peak over nodes at offset 0.  These decide which CPU
kernel the reference runtime runs for the baseline, so they must agree with it.

For the CUDA target (backend `delegate`) the tokens map to device kernels:
  Conv  cuda_tc_int8   -> tc_int8    (tcgen05 kind::i8, int8 weights)
        cuda_tc_3xtf32 -> tc_3xtf32  (tcgen05 kind::tf32, 3xTF32 split)
        cuda_tc_tf32   -> tc_tf32    (tcgen05 kind::tf32, plain)
        cuda_simt_fp32 -> simt_fp32  (CUDA-core FFMA)
  Gemm  cuda_direct    -> direct
  other cuda           -> reference  (the op's CUDA kernel)
CUDA specs carry layout NHWC (the device activation layout), need no SPK
scratch, and have no fallback: the profile lists no `ref` token.

Weight pre-packing (the reference format's weight_layout field,
reference compiler/planner/kernel_spec.py:43, packager/spk_writer.py:35): a
tensor-core fp32 conv whose weights the device reads as they are packed gets
weight_layout TC_PANEL_F32X2 and the SPK writer stores its weights as the
tcgen05 operand panel (see spk_writer.tc_panel), so prepare on the device is
an upload with no repacking.  Eligible: fp32 weights, group 1, Cout >= 16,
Cin a multiple of 4 above 4 (the device then keeps Cin as the GEMM channel
count whatever the input layout; few-channel first convs are row-packed at
prepare and keep OIHW).
"""

from __future__ import annotations

from dataclasses import dataclass

from .ir import DTYPE_FP32, DTYPE_INT8, Graph, Node

BACKEND_REF, BACKEND_CPU, BACKEND_SIMD, BACKEND_DELEGATE = "ref", "cpu", "simd", "delegate"

KIND_REFERENCE = "reference"
KIND_DIRECT = "direct"
KIND_IM2COL_GEMM = "im2col_gemm"
KIND_POINTWISE_1X1 = "pointwise_1x1"
KIND_DEPTHWISE_DIRECT = "depthwise_direct"
KIND_WINOGRAD_3X3S1 = "winograd_3x3s1"
KIND_WINOGRAD_F43 = "winograd_f43"
KIND_CONV3X3S2_DIRECT = "conv3x3s2_direct"
KIND_INT8_IM2COL_GEMM = "int8_im2col_gemm"
KIND_BNNS_FP32 = "bnns_fp32"
KIND_TC_3XTF32 = "tc_3xtf32"
KIND_TC_TF32 = "tc_tf32"
KIND_TC_INT8 = "tc_int8"
KIND_SIMT_FP32 = "simt_fp32"

WEIGHT_LAYOUT_OIHW = "OIHW"
WEIGHT_LAYOUT_TC_PANEL = "TC_PANEL_F32X2"

SIMD_TILE_BYTES = 32 * 1024 * 1024  # cap of the CPU SIMD conv's working buffers
SIMD_IM2COL_SEGMENT = 2 * 1024 * 1024

CUDA_CONV_TOKENS = {
    "cuda_tc_int8": KIND_TC_INT8,
    "cuda_tc_3xtf32": KIND_TC_3XTF32,
    "cuda_tc_tf32": KIND_TC_TF32,
    "cuda_simt_fp32": KIND_SIMT_FP32,
}

SIMD_ELEMENTWISE_OPS = {
    "Add", "Mul", "Sub", "Div", "Relu", "Sigmoid", "Transpose", "ReduceMax", "ReduceMean", "Softmax",
    "MaxPool", "Resize", "AveragePool", "GlobalAveragePool", "Clip", "LeakyRelu",
}


@dataclass
class KernelSpec:
    id: int
    node_id: int
    op_type: str
    kernel_kind: str
    backend: str
    dtype: str = DTYPE_FP32
    layout: str = "NCHW"
    weight_layout: str = "OIHW"
    scratch_offset: int = 0
    scratch_bytes: int = 0
    fallback_kernel_spec_id: int = 0xFFFFFFFF
    required_features: list[str] | None = None
    selected_by_fallback: bool = False


@dataclass
class KernelPlan:
    specs: list[KernelSpec]
    by_node: dict[int, KernelSpec]
    scratch_arena_bytes: int
    fallback_count: int


def select_kernel_specs(graph: Graph, profile: dict) -> KernelPlan:
    specs: list[KernelSpec] = []
    by_node: dict[int, KernelSpec] = {}
    fallbacks = 0
    peak = 0
    for node in graph.nodes:
        tokens = profile["ops"].get(node.op_type, [])
        if not tokens:
            raise ValueError(f"target profile does not support op: {node.op_type}")
        chosen = _primary(graph, node, tokens, profile)
        ref_spec = _spec(graph, node, KIND_REFERENCE, BACKEND_REF)
        if chosen is None:
            if "ref" not in tokens:
                raise ValueError(f"no supported kernel for op: {node.op_type}")
            chosen = ref_spec
            chosen.selected_by_fallback = True
            fallbacks += 1
        chosen.id = len(specs)
        specs.append(chosen)
        by_node[node.id] = chosen
        if chosen.kernel_kind != KIND_REFERENCE and "ref" in tokens:
            ref_spec.id = len(specs)
            chosen.fallback_kernel_spec_id = ref_spec.id
            specs.append(ref_spec)
        peak = max(peak, chosen.scratch_bytes)
    limit = int(profile["memory"]["scratch_arena_max"])
    if peak > limit:
        raise MemoryError(f"planned scratch arena {peak} exceeds target limit {limit}")
    graph.metadata["kernel_specs"] = [_spec_json(s) for s in specs]
    graph.metadata["kernel_fallback_count"] = fallbacks
    graph.metadata["scratch_arena_bytes"] = peak
    return KernelPlan(specs, by_node, peak, fallbacks)


def _primary(graph: Graph, node: Node, tokens: list[str], profile: dict) -> KernelSpec | None:
    if any(t.startswith("cuda") for t in tokens):
        return _primary_cuda(graph, node, tokens, "TC_PANEL_F32X2" in profile.get("weight_layouts", []))
    if node.op_type == "Conv":
        if len(node.inputs) > 1:
            w = graph.tensors[node.inputs[1]]
            if w.dtype == DTYPE_INT8 and int(node.attrs.get("group", 1)) == 1 and "simd_int8_im2col_gemm" in tokens:
                return _spec(graph, node, KIND_INT8_IM2COL_GEMM, BACKEND_SIMD, dtype=DTYPE_INT8)
        kind = _simd_conv_kind(graph, node, tokens)
        if kind is not None:
            return _spec(graph, node, kind, BACKEND_SIMD)
    if node.op_type in ("Gemm", "MatMul") and "simd_direct" in tokens:
        return _spec(graph, node, KIND_DIRECT, BACKEND_SIMD)
    if "simd" in tokens and node.op_type in SIMD_ELEMENTWISE_OPS:
        return _spec(graph, node, KIND_REFERENCE, BACKEND_SIMD)
    if node.op_type == "Conv" and KIND_IM2COL_GEMM in tokens:
        return _spec(graph, node, KIND_IM2COL_GEMM, BACKEND_CPU)
    if node.op_type == "Gemm" and KIND_DIRECT in tokens:
        return _spec(graph, node, KIND_DIRECT, BACKEND_CPU)
    if KIND_REFERENCE in tokens or "ref" in tokens:
        return _spec(graph, node, KIND_REFERENCE, BACKEND_REF)
    return None


def _primary_cuda(graph: Graph, node: Node, tokens: list[str], prepack: bool = False) -> KernelSpec | None:
    if node.op_type == "Conv":
        w = graph.tensors[node.inputs[1]]
        for tok in tokens:
            kind = CUDA_CONV_TOKENS.get(tok)
            if kind is None:
                continue
            if (kind == KIND_TC_INT8) != (w.dtype == DTYPE_INT8):
                continue
            spec = _spec(graph, node, kind, BACKEND_DELEGATE, dtype=w.dtype, layout="NHWC")
            if prepack and tc_panel_eligible(graph, node, kind):
                spec.weight_layout = WEIGHT_LAYOUT_TC_PANEL
            return spec
        return None
    if node.op_type == "Gemm" and "cuda_direct" in tokens:
        return _spec(graph, node, KIND_DIRECT, BACKEND_DELEGATE, layout="NHWC")
    if "cuda" in tokens:
        return _spec(graph, node, KIND_REFERENCE, BACKEND_DELEGATE, layout="NHWC")
    return None


def tc_panel_eligible(graph: Graph, node: Node, kind: str) -> bool:
    """A Conv whose fp32 weights the tcgen05 kernels read in the panel layout
    the SPK writer can produce ahead of time (see the module docstring)."""
    if kind not in (KIND_TC_3XTF32, KIND_TC_TF32) or len(node.inputs) < 2:
        return False
    w = graph.tensors[node.inputs[1]]
    if w.dtype != DTYPE_FP32 or len(w.shape) != 4 or w.data is None:
        return False
    if int(node.attrs.get("group", 1)) != 1:
        return False
    cout, cin = int(w.shape[0]), int(w.shape[1])
    out = graph.tensors[node.outputs[0]] if node.outputs else None
    return cout >= 16 and cin % 4 == 0 and cin > 4 and out is not None and out.dtype == DTYPE_FP32


def _ints(value, length: int, default: int) -> list[int]:
    out = [int(v) for v in value]
    return (out + [default] * length)[:length]


def _simd_conv_kind(graph: Graph, node: Node, tokens: list[str]) -> str | None:
    x = graph.tensors[node.inputs[0]] if node.inputs else None
    w = graph.tensors[node.inputs[1]] if len(node.inputs) > 1 else None
    if x is None or w is None or len(x.shape) != 4 or len(w.shape) != 4:
        return KIND_IM2COL_GEMM if "simd_im2col_gemm" in tokens else None
    group = int(node.attrs.get("group", 1))
    strides = _ints(node.attrs.get("strides", [1, 1]), 2, 1)
    pads = _ints(node.attrs.get("pads", [0, 0, 0, 0]), 4, 0)
    dil = _ints(node.attrs.get("dilations", [1, 1]), 2, 1)
    kh, kw = int(w.shape[2]), int(w.shape[3])
    cin, cout = int(x.shape[1]), int(w.shape[0])
    if "simd_bnns_fp32" in tokens and group == 1:
        return KIND_BNNS_FP32
    if ("simd_pointwise_1x1" in tokens and group == 1 and (kh, kw) == (1, 1) and strides == [1, 1]
            and pads == [0, 0, 0, 0] and dil == [1, 1]):
        return KIND_POINTWISE_1X1
    if ("simd_depthwise_direct" in tokens and group == cin and group == cout and (kh, kw) == (3, 3)
            and dil == [1, 1]):
        return KIND_DEPTHWISE_DIRECT
    if ("simd_winograd_f43" in tokens and group == 1 and (kh, kw) == (3, 3) and strides == [1, 1]
            and dil == [1, 1] and pads == [1, 1, 1, 1]):
        y = graph.tensors[node.outputs[0]]
        if len(y.shape) == 4:
            oh, ow = int(y.shape[2]), int(y.shape[3])
            tiles = ((oh + 3) // 4) * ((ow + 3) // 4)
            if (oh >= 8 and ow >= 8 and (cin >= 8 or cout >= 8) and tiles >= 4
                    and 36 * (cin + cout) * tiles * 4 <= SIMD_TILE_BYTES):
                return KIND_WINOGRAD_F43
    if ("simd_conv3x3s2_direct" in tokens and group == 1 and (kh, kw) == (3, 3) and strides == [2, 2]
            and dil == [1, 1] and pads == [1, 1, 1, 1]):
        return KIND_CONV3X3S2_DIRECT
    if "simd_im2col_gemm" in tokens:
        return KIND_IM2COL_GEMM
    return None


def _spec(graph: Graph, node: Node, kind: str, backend: str, dtype: str = DTYPE_FP32,
          layout: str = "NCHW") -> KernelSpec:
    return KernelSpec(id=0, node_id=node.id, op_type=node.op_type, kernel_kind=kind, backend=backend, dtype=dtype,
                      layout=layout, scratch_bytes=_scratch(graph, node, kind, backend), required_features=[dtype])


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def _scratch(graph: Graph, node: Node, kind: str, backend: str) -> int:
    if node.op_type != "Conv" or backend == BACKEND_DELEGATE:
        return 0
    if kind in (KIND_POINTWISE_1X1, KIND_DEPTHWISE_DIRECT, KIND_CONV3X3S2_DIRECT, KIND_BNNS_FP32):
        return 0
    x = graph.tensors[node.inputs[0]]
    w = graph.tensors[node.inputs[1]]
    y = graph.tensors[node.outputs[0]]
    if kind in (KIND_WINOGRAD_3X3S1, KIND_WINOGRAD_F43):
        if len(x.shape) != 4 or len(w.shape) != 4 or len(y.shape) != 4:
            return 0
        step, width = (2, 16) if kind == KIND_WINOGRAD_3X3S1 else (4, 36)
        tiles = ((y.shape[2] + step - 1) // step) * ((y.shape[3] + step - 1) // step)
        return _align(min(width * (x.shape[1] + w.shape[0]) * tiles * 4, SIMD_TILE_BYTES), 16)
    if kind == KIND_INT8_IM2COL_GEMM:
        if len(x.shape) != 4 or len(w.shape) != 4 or len(y.shape) != 4:
            return 0
        k = x.shape[1] * w.shape[2] * w.shape[3]
        spatial = y.shape[2] * y.shape[3]
        return _align(x.shape[1] * x.shape[2] * x.shape[3] + k * spatial + w.shape[0] * spatial * 4, 16)
    if kind != KIND_IM2COL_GEMM or len(x.shape) != 4 or len(w.shape) != 4:
        return 0
    k = x.shape[1] * w.shape[2] * w.shape[3]
    if backend == BACKEND_SIMD:
        spatial = y.shape[2] * y.shape[3] if len(y.shape) == 4 else 1
        return _align(min(k * spatial * 4, SIMD_IM2COL_SEGMENT), 16)
    return _align(k * 4, 16)


def _spec_json(spec: KernelSpec) -> dict:
    return {
        "id": spec.id, "node_id": spec.node_id, "op_type": spec.op_type, "kernel_kind": spec.kernel_kind,
        "backend": spec.backend, "dtype": spec.dtype, "layout": spec.layout, "weight_layout": spec.weight_layout,
        "scratch_offset": spec.scratch_offset, "scratch_bytes": spec.scratch_bytes,
        "fallback_kernel_spec_id": spec.fallback_kernel_spec_id,
        "required_features": spec.required_features or [], "selected_by_fallback": spec.selected_by_fallback,
    }
