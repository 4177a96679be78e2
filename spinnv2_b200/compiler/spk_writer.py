"""SPK v0.3 package writer.

Binary layout (little-endian, packed) is the SPK format that SPINNV2's runtime
loads (reference compiler/packager/spk_writer.py:99-200, format/spk_format.md):
header, section directory, then sections in the order metadata, target
profile, tensor table, node table, attributes, weights (4096-byte aligned,
each weight 16-byte aligned), memory plan, kernel specs, [quantisation],
[protection], string table, checksum.  The checksum is FNV-1a 32 over every
byte before the checksum section.

Codes added by the CUDA target (unused values in the reference's tables):
dtype int32 = 4 (the int32 bias of INT8 convs), kernel kinds tc_3xtf32 = 12,
tc_tf32 = 13, tc_int8 = 14, simt_fp32 = 15, layout NHWC = 2.
"""

from __future__ import annotations

import ctypes
import json
import struct
from pathlib import Path

import numpy as np

from .ir import DTYPE_FP16, DTYPE_FP32, DTYPE_INT8, DTYPE_INT32, ROLE_ACTIVATION, ROLE_CONSTANT, ROLE_INPUT, \
    ROLE_OUTPUT, ROLE_WEIGHT, Graph, Node
from .kernel_spec import KernelPlan, KernelSpec, select_kernel_specs
from .memory_plan import MemoryPlan, plan_for_profile

SPKV2_MAGIC = 0x32564B50
VERSION_MAJOR, VERSION_MINOR = 0, 3

SECTION_METADATA = 1
SECTION_TARGET_PROFILE = 2
SECTION_TENSOR_TABLE = 3
SECTION_NODE_TABLE = 4
SECTION_ATTRIBUTES = 5
SECTION_WEIGHTS = 6
SECTION_MEMORY_PLAN = 7
SECTION_KERNEL_SPEC = 8
SECTION_QUANTIZATION = 9
SECTION_STRING_TABLE = 10
SECTION_CHECKSUM = 12
SECTION_PROTECTION_PLAN = 13

DTYPE_CODES = {DTYPE_FP32: 1, DTYPE_INT8: 2, DTYPE_FP16: 3, DTYPE_INT32: 4}
LAYOUT_CODES = {"NCHW": 1, "NHWC": 2}
WEIGHT_LAYOUT_CODES = {"OIHW": 1, "TC_PANEL_F32X2": 2}
TC_PANEL_N_ALIGN = 256  # panel rows padded for every tile width the device may pick (32..256)
TC_PANEL_K_ALIGN = 32   # one K step of the fp32 tcgen05 kernels


def tc_panel(w: np.ndarray) -> np.ndarray:
    """fp32 OIHW conv weights [M, C, KH, KW] -> the tcgen05 operand panel
    [2][Npad][Kpad] (K-major rows, k = (r * KW + s) * C + c, zero padding;
    Npad = M rounded up to 256, Kpad = K rounded up to 32).  Part 0 is each
    weight rounded to TF32 (10 mantissa bits, to nearest, ties away from
    zero), part 1 the remainder w - part0, exact in fp32, so part0 + part1
    == w bit for bit and the 3xTF32 kernels read both parts as stored."""
    m, c, kh, kw = w.shape
    k = c * kh * kw
    npad = -(-m // TC_PANEL_N_ALIGN) * TC_PANEL_N_ALIGN
    kpad = -(-k // TC_PANEL_K_ALIGN) * TC_PANEL_K_ALIGN
    wk = np.ascontiguousarray(np.asarray(w, dtype=np.float32).transpose(0, 2, 3, 1)).reshape(m, k)
    bits = wk.view(np.uint32)
    finite = (bits & np.uint32(0x7F800000)) != np.uint32(0x7F800000)
    hi_bits = np.where(finite, (bits + np.uint32(0x1000)) & np.uint32(0xFFFFE000), bits)
    hi = hi_bits.view(np.float32)
    lo = (wk - hi).astype(np.float32)
    panel = np.zeros((2, npad, kpad), dtype=np.float32)
    panel[0, :m, :k] = hi
    panel[1, :m, :k] = lo
    return panel


def tc_panel_to_oihw(panel: np.ndarray, shape) -> np.ndarray:
    """Inverse of tc_panel: the OIHW weights (part0 + part1, exact)."""
    m, c, kh, kw = (int(d) for d in shape)
    k = c * kh * kw
    wk = (panel[0, :m, :k] + panel[1, :m, :k]).astype(np.float32)
    return np.ascontiguousarray(wk.reshape(m, kh, kw, c).transpose(0, 3, 1, 2))
BACKEND_CODES = {"ref": 1, "cpu": 2, "simd": 3, "delegate": 4}
KERNEL_KIND_CODES = {
    "reference": 1, "direct": 2, "im2col_gemm": 3, "packed_gemm": 4, "pointwise_1x1": 5,
    "depthwise_direct": 6, "winograd_3x3s1": 7, "conv3x3s2_direct": 8, "winograd_f43": 9,
    "int8_im2col_gemm": 10, "bnns_fp32": 11,
    "tc_3xtf32": 12, "tc_tf32": 13, "tc_int8": 14, "simt_fp32": 15,
}
ROLE_CODES = {ROLE_INPUT: 1, ROLE_OUTPUT: 2, ROLE_WEIGHT: 3, ROLE_ACTIVATION: 4, ROLE_CONSTANT: 5}
MEMORY_CLASS_CODES = {"INPUT": 1, "OUTPUT": 2, "WEIGHT": 3, "ACTIVATION_ARENA": 4, "EXTERNAL": 5}
OP_CODES = {
    "Add": 1, "Conv": 2, "Flatten": 3, "Gemm": 4, "MaxPool": 5, "Relu": 6, "Softmax": 7, "Mul": 8,
    "Sub": 9, "Div": 10, "Mod": 11, "Sigmoid": 12, "Reshape": 13, "Transpose": 14, "Concat": 15,
    "Split": 16, "ReduceMean": 17, "ReduceMax": 18, "MatMul": 19, "Resize": 20, "Tile": 21,
    "Unsqueeze": 22, "GatherElements": 23, "TopK": 24, "Cast": 25, "Slice": 26, "Gather": 27,
    "AveragePool": 28, "GlobalAveragePool": 29, "Clip": 30, "LeakyRelu": 31,
}
ACTIVATION_CODES = {"Relu": 1, "Silu": 2}
QUANT_SCHEME_CODES = {"per_tensor": 1, "per_channel": 2}

HEADER = struct.Struct("<IHHHHIIIIIIQQQII")
SECTION = struct.Struct("<IIQQII")
TENSOR = struct.Struct("<IHHHH8IQQII")
NODE = struct.Struct("<IHHHH8I4IIIII")
ATTR = struct.Struct("<Iiii4i2i2i2i2i2fii8i3i")
MEMORY_PLAN = struct.Struct("<IHHIQQII")
KERNEL_SPEC = struct.Struct("<IIHHHHHHQQII")
QUANT_PARAM = struct.Struct("<IHHIQ")


# Large packages take the runtime library's C loop for their checksum unless
# this is False (then the pure-Python loop, as the reference compiler does;
# a process that must not map the CUDA library sets it).
NATIVE_FNV = True


def fnv1a32(data: bytes | bytearray | memoryview) -> int:
    """FNV-1a 32-bit; uses the runtime library's C loop for large packages."""
    if NATIVE_FNV and len(data) > (1 << 16):
        fn = _native_fnv()
        if fn is not None:
            buf = (ctypes.c_char * len(data)).from_buffer_copy(data) if isinstance(data, bytes) else \
                (ctypes.c_char * len(data)).from_buffer(data)
            return int(fn(buf, len(data)))
    h = 0x811C9DC5
    for b in bytes(data):
        h = ((h ^ b) * 0x01000193) & 0xFFFFFFFF
    return h


_FNV = None


def _native_fnv():
    global _FNV
    if _FNV is None:
        try:
            from ..runtime import load_library
            lib = load_library()
            fn = lib.spkv2_fnv1a32
            fn.restype = ctypes.c_uint32
            fn.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
            _FNV = fn
        except Exception:  # library not built yet: pure-Python loop
            _FNV = False
    return _FNV or None


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def _ints(value, length: int, default: int) -> list[int]:
    out = [int(v) for v in value]
    return (out + [default] * length)[:length]


def attr_bytes(node: Node) -> bytes:
    a = node.attrs
    kernel = _ints(a.get("kernel_shape", [1, 1]), 2, 1)
    strides = _ints(a.get("strides", [1, 1]), 2, 1)
    pads = _ints(a.get("pads", [0, 0, 0, 0]), 4, 0)
    dil = _ints(a.get("dilations", [1, 1]), 2, 1)
    extra: list[int] = []
    if node.op_type == "Transpose":
        extra = [int(v) for v in a.get("perm", [])]
    elif node.op_type in ("ReduceMean", "ReduceMax") and "axes" in a:
        extra = [int(v) for v in a.get("axes", [])]
    return ATTR.pack(
        OP_CODES[node.op_type], int(a.get("axis", 1)), int(a.get("group", 1)),
        ACTIVATION_CODES.get(a.get("fused_activation"), 0), *pads, *strides, *kernel, *dil,
        int(a.get("transA", 0)), int(a.get("transB", 0)), float(a.get("alpha", 1.0)), float(a.get("beta", 1.0)),
        len(extra), int(a.get("keepdims", 1)), *((extra + [0] * 8)[:8]), int(a.get("largest", 1)),
        int(a.get("sorted", 1)), int(a.get("to", 1)))


def build_spk(graph: Graph, profile: dict, *, memory_plan: MemoryPlan | None = None,
              kernel_plan: KernelPlan | None = None, quant_params: list | None = None,
              protection_plan=None) -> tuple[bytes, dict]:
    """Serialise `graph` for `profile`; returns (package bytes, debug dict).
    `protection_plan` (compiler.protection.ProtectionPlan) adds the protection
    section after the quantisation section and grows the scratch arena by
    its DMR copies (reference compiler/packager/spk_writer.py:147-149,187)."""
    unknown = sorted({n.op_type for n in graph.nodes if n.op_type not in OP_CODES})
    if unknown:
        raise ValueError(f"graph still contains unsupported runtime op(s): {', '.join(unknown)}")
    if kernel_plan is None:
        kernel_plan = select_kernel_specs(graph, profile)
    if memory_plan is None:
        memory_plan = plan_for_profile(graph, profile)

    strings = bytearray(b"\x00")
    name_off: dict[str, int] = {"": 0}
    for t in graph.tensors:
        if t.name not in name_off:
            name_off[t.name] = len(strings)
            strings.extend(t.name.encode("utf-8") + b"\x00")

    # Weights the kernel plan asks for pre-packed (weight_layout) are stored
    # in that layout; their records keep the logical shape and give the
    # stored byte size.
    panel_of = {}
    for n in graph.nodes:
        if kernel_plan.by_node[n.id].weight_layout == "TC_PANEL_F32X2":
            panel_of[n.inputs[1]] = True
    weights = bytearray()
    weight_off: dict[int, int] = {}
    weight_size: dict[int, int] = {}
    for t in graph.tensors:
        if t.role != ROLE_WEIGHT:
            continue
        if t.data is None:
            raise ValueError(f"weight tensor missing data: {t.name}")
        weights.extend(b"\x00" * (_align(len(weights), 16) - len(weights)))
        weight_off[t.id] = len(weights)
        blob = tc_panel(t.array()).tobytes() if t.id in panel_of else t.data
        weight_size[t.id] = len(blob)
        weights.extend(blob)

    attrs = bytearray()
    attr_off: dict[int, tuple[int, int]] = {}
    for n in graph.nodes:
        attrs.extend(b"\x00" * (_align(len(attrs), 4) - len(attrs)))
        blob = attr_bytes(n)
        attr_off[n.id] = (len(attrs), len(blob))
        attrs.extend(blob)

    tensors = bytearray()
    for t in graph.tensors:
        e = memory_plan.entries[t.id]
        tensors.extend(TENSOR.pack(t.id, DTYPE_CODES[t.dtype], ROLE_CODES[t.role], len(t.shape),
                                   MEMORY_CLASS_CODES[e.memory_class], *(t.shape[:8] + [1] * (8 - len(t.shape))),
                                   weight_size.get(t.id, t.size_bytes), weight_off.get(t.id, e.offset),
                                   name_off[t.name], 0))
    nodes = bytearray()
    for n in graph.nodes:
        spec = kernel_plan.by_node[n.id]
        ao, asz = attr_off[n.id]
        nodes.extend(NODE.pack(n.id, OP_CODES[n.op_type], 0, len(n.inputs), len(n.outputs),
                               *(n.inputs[:8] + [0] * (8 - len(n.inputs))),
                               *(n.outputs[:4] + [0] * (4 - len(n.outputs))), ao, asz, spec.id, spec.scratch_bytes))
    plan = bytearray()
    for t in graph.tensors:
        e = memory_plan.entries[t.id]
        plan.extend(MEMORY_PLAN.pack(e.tensor_id, MEMORY_CLASS_CODES[e.memory_class], 16, 0, e.offset, e.size,
                                     e.first_use if e.first_use >= 0 else 0xFFFFFFFF,
                                     e.last_use if e.last_use >= 0 else 0xFFFFFFFF))
    specs = bytearray()
    for s in kernel_plan.specs:
        specs.extend(_spec_bytes(s))

    metadata = json.dumps({"model_name": graph.model_name, "sir_version": "0.1", "inputs": graph.inputs,
                           "outputs": graph.outputs}, sort_keys=True).encode("utf-8")
    sections: list[tuple[int, bytes, int]] = [
        (SECTION_METADATA, metadata, 1),
        (SECTION_TARGET_PROFILE, json.dumps(profile, sort_keys=True).encode("utf-8"), 1),
        (SECTION_TENSOR_TABLE, bytes(tensors), 4),
        (SECTION_NODE_TABLE, bytes(nodes), 4),
        (SECTION_ATTRIBUTES, bytes(attrs), 4),
        (SECTION_WEIGHTS, bytes(weights), 4096),
        (SECTION_MEMORY_PLAN, bytes(plan), 4),
        (SECTION_KERNEL_SPEC, bytes(specs), 4),
    ]
    if quant_params:
        sections.append((SECTION_QUANTIZATION, quantization_section(quant_params), 4))
    prot_scratch = 0
    if protection_plan is not None:
        sections.append((SECTION_PROTECTION_PLAN,
                         protection_plan.section(graph, scratch_offset=kernel_plan.scratch_arena_bytes), 8))
        prot_scratch = protection_plan.scratch_bytes(graph)
    sections.append((SECTION_STRING_TABLE, bytes(strings), 1))
    sections.append((SECTION_CHECKSUM, b"\x00\x00\x00\x00", 4))

    offset = HEADER.size + len(sections) * SECTION.size
    directory = bytearray()
    payload = bytearray()
    checksum_at = 0
    for kind, data, alignment in sections:
        aligned = _align(offset, alignment)
        payload.extend(b"\x00" * (aligned - offset))
        offset = aligned
        if kind == SECTION_CHECKSUM:
            checksum_at = offset
        directory.extend(SECTION.pack(kind, 0, offset, len(data), alignment, 0))
        payload.extend(data)
        offset += len(data)
    header = HEADER.pack(SPKV2_MAGIC, VERSION_MAJOR, VERSION_MINOR, 0, HEADER.size, len(sections), 0,
                         len(graph.tensors), len(graph.nodes), len(graph.inputs), len(graph.outputs),
                         sum(weight_size.values()),
                         memory_plan.planned_activation_bytes, kernel_plan.scratch_arena_bytes + prot_scratch,
                         fnv1a32(json.dumps(profile, sort_keys=True).encode("utf-8")), 1)
    package = bytearray(header + directory + payload)
    package[checksum_at:checksum_at + 4] = struct.pack("<I", fnv1a32(memoryview(package)[:checksum_at]))
    return bytes(package), _debug(graph, memory_plan)


def write_spk(graph: Graph, out_path: str | Path, profile: dict, **kw) -> Path:
    out_path = Path(out_path)
    data, debug = build_spk(graph, profile, **kw)
    out_path.parent.mkdir(parents=True, exist_ok=True)
    out_path.write_bytes(data)
    out_path.with_suffix(out_path.suffix + ".json").write_text(json.dumps(debug, indent=2, default=str),
                                                               encoding="utf-8")
    return out_path


def _spec_bytes(s: KernelSpec) -> bytes:
    mask = (1 if DTYPE_FP32 in (s.required_features or []) else 0) | \
           (2 if DTYPE_INT8 in (s.required_features or []) else 0) | \
           (4 if DTYPE_FP16 in (s.required_features or []) else 0)
    return KERNEL_SPEC.pack(s.id, s.node_id, KERNEL_KIND_CODES[s.kernel_kind], BACKEND_CODES[s.backend],
                            DTYPE_CODES[s.dtype], LAYOUT_CODES[s.layout], WEIGHT_LAYOUT_CODES[s.weight_layout], 0,
                            s.scratch_offset, s.scratch_bytes, s.fallback_kernel_spec_id, mask)


def quantization_section(quant_params: list) -> bytes:
    """Records first, then per record float scales and int32 zero points."""
    records_size = len(quant_params) * QUANT_PARAM.size
    data = bytearray()
    offsets = []
    for qp in quant_params:
        offsets.append(records_size + len(data))
        data.extend(struct.pack(f"<{len(qp.scales)}f", *qp.scales))
        data.extend(struct.pack(f"<{len(qp.zero_points)}i", *qp.zero_points))
    records = bytearray()
    for qp, off in zip(quant_params, offsets):
        records.extend(QUANT_PARAM.pack(qp.tensor_id, QUANT_SCHEME_CODES.get(qp.scheme, 0), qp.quant_axis,
                                        qp.num_channels, off))
    return bytes(records + data)


def _debug(graph: Graph, plan: MemoryPlan) -> dict:
    return {
        "model_name": graph.model_name,
        "inputs": graph.inputs,
        "outputs": graph.outputs,
        "metadata": graph.metadata,
        "memory": {
            "naive_activation_bytes": plan.naive_activation_bytes,
            "planned_activation_bytes": plan.planned_activation_bytes,
            "memory_reduction_ratio": plan.memory_reduction_ratio,
        },
        "nodes": [{"id": n.id, "op_type": n.op_type, "inputs": n.inputs, "outputs": n.outputs, "attrs": n.attrs}
                  for n in graph.nodes],
    }
