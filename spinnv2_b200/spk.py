"""Read an SPK v0.3 package into Python structures.

Parses the same records the C loader maps (reference runtime/core/loader.c:
140-282; layouts in include/spkv2_format.h): tensors, nodes with decoded
attributes, kernel specs, memory plan, quantisation parameters and weights.
Used by the ctypes driver (output shapes/dtypes), the tests and the CPU
oracle harness.
"""

from __future__ import annotations

import functools
import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .compiler import spk_writer as W

DTYPE_NAMES = {1: "fp32", 2: "int8", 3: "fp16", 4: "int32"}
NUMPY_OF = {1: np.float32, 2: np.int8, 3: np.float16, 4: np.int32}
OP_NAMES = {v: k for k, v in W.OP_CODES.items()}
KIND_NAMES = {v: k for k, v in W.KERNEL_KIND_CODES.items()}
BACKEND_NAMES = {v: k for k, v in W.BACKEND_CODES.items()}
ROLE_NAMES = {v: k for k, v in W.ROLE_CODES.items()}


@dataclass
class SpkTensor:
    id: int
    dtype: int
    role: int
    shape: list[int]
    memory_class: int
    size_bytes: int
    data_offset: int
    name: str

    @property
    def np_dtype(self):
        return NUMPY_OF[self.dtype]

    @property
    def role_name(self) -> str:
        return ROLE_NAMES[self.role]


@dataclass
class SpkAttr:
    axis: int
    group: int
    fused_activation: int
    pads: list[int]
    strides: list[int]
    kernel_shape: list[int]
    dilations: list[int]
    trans_a: int
    trans_b: int
    alpha: float
    beta: float
    extra: list[int]
    keepdims: int
    largest: int
    sorted: int
    cast_to: int


@dataclass
class SpkNode:
    id: int
    op_type: str
    inputs: list[int]
    outputs: list[int]
    attr: SpkAttr | None
    kernel_spec_id: int
    scratch_bytes: int


@dataclass
class SpkKernelSpec:
    id: int
    node_id: int
    kind: str
    backend: str
    dtype: int
    layout: int
    scratch_bytes: int
    fallback: int
    weight_layout: int = 1  # 1 OIHW, 2 the tcgen05 panel (spk_writer.tc_panel)


@dataclass
class SpkQuant:
    tensor_id: int
    scheme: int
    axis: int
    scales: np.ndarray
    zero_points: np.ndarray


@dataclass
class SpkPackage:
    header: dict
    tensors: list[SpkTensor]
    nodes: list[SpkNode]
    specs: list[SpkKernelSpec]
    quant: dict[int, SpkQuant]
    weights: bytes
    metadata: dict
    profile: dict
    plan: list[tuple] = field(default_factory=list)

    @property
    def inputs(self) -> list[SpkTensor]:
        return [t for t in self.tensors if t.role == 1]

    @property
    def outputs(self) -> list[SpkTensor]:
        order = self.metadata.get("outputs")
        outs = [t for t in self.tensors if t.role == 2]
        if order and len(order) == len(outs):
            return [self.tensors[i] for i in order]
        return outs

    @functools.cached_property
    def panel_weights(self) -> frozenset[int]:
        """Ids of the weight tensors stored pre-packed as tcgen05 panels."""
        return frozenset(n.inputs[1] for n in self.nodes
                if n.op_type == "Conv" and n.kernel_spec_id < len(self.specs)
                         and self.specs[n.kernel_spec_id].weight_layout == 2)

    def weight(self, tid: int) -> np.ndarray:
        """A weight tensor in its logical (OIHW / row-major) layout; panels
        written pre-packed are unpacked (exactly: part0 + part1 == w)."""
        t = self.tensors[tid]
        buf = self.weights[t.data_offset:t.data_offset + t.size_bytes]
        if tid in self.panel_weights:
            m, c, kh, kw = t.shape
            npad = -(-m // W.TC_PANEL_N_ALIGN) * W.TC_PANEL_N_ALIGN
            kpad = -(-(c * kh * kw) // W.TC_PANEL_K_ALIGN) * W.TC_PANEL_K_ALIGN
            panel = np.frombuffer(buf, dtype=np.float32).reshape(2, npad, kpad)
            return W.tc_panel_to_oihw(panel, t.shape)
        return np.frombuffer(buf, dtype=t.np_dtype).reshape(t.shape)


def read_spk(src: str | Path | bytes) -> SpkPackage:
    data = Path(src).read_bytes() if not isinstance(src, (bytes, bytearray)) else bytes(src)
    h = W.HEADER.unpack_from(data, 0)
    keys = ["magic", "version_major", "version_minor", "endianness", "header_size", "section_count", "model_flags",
            "num_tensors", "num_nodes", "num_inputs", "num_outputs", "weight_bytes", "activation_arena_bytes",
            "scratch_arena_bytes", "target_profile_hash", "checksum_type"]
    header = dict(zip(keys, h))
    if header["magic"] != W.SPKV2_MAGIC:
        raise ValueError("not an SPK package")
    sections = {}
    for i in range(header["section_count"]):
        kind, _flags, off, size, _al, _r = W.SECTION.unpack_from(data, header["header_size"] + i * W.SECTION.size)
        sections[kind] = (off, size)

    def sec(kind):
        off, size = sections.get(kind, (0, 0))
        return data[off:off + size]

    strings = sec(W.SECTION_STRING_TABLE)

    def name_at(o: int) -> str:
        end = strings.find(b"\x00", o)
        return strings[o:end].decode("utf-8")

    tensors = []
    tt = sec(W.SECTION_TENSOR_TABLE)
    for i in range(header["num_tensors"]):
        f = W.TENSOR.unpack_from(tt, i * W.TENSOR.size)
        rank = f[3]
        tensors.append(SpkTensor(f[0], f[1], f[2], list(f[5:5 + rank]), f[4], f[13], f[14], name_at(f[15])))
    attrs_blob = sec(W.SECTION_ATTRIBUTES)
    nodes = []
    nt = sec(W.SECTION_NODE_TABLE)
    for i in range(header["num_nodes"]):
        f = W.NODE.unpack_from(nt, i * W.NODE.size)
        nid, op, _flags, nin, nout = f[:5]
        ins = list(f[5:5 + nin])
        outs = list(f[13:13 + nout])
        aoff, asz, spec_id, scratch = f[17:21]
        attr = None
        if asz >= W.ATTR.size:
            a = W.ATTR.unpack_from(attrs_blob, aoff)
            attr = SpkAttr(axis=a[1], group=a[2], fused_activation=a[3], pads=list(a[4:8]), strides=list(a[8:10]),
                           kernel_shape=list(a[10:12]), dilations=list(a[12:14]), trans_a=a[14], trans_b=a[15],
                           alpha=a[16], beta=a[17], extra=list(a[20:20 + max(0, min(8, a[18]))]), keepdims=a[19],
                           largest=a[28], sorted=a[29], cast_to=a[30])
        nodes.append(SpkNode(nid, OP_NAMES.get(op, f"op{op}"), ins, outs, attr, spec_id, scratch))
    specs = []
    ks = sec(W.SECTION_KERNEL_SPEC)
    for i in range(len(ks) // W.KERNEL_SPEC.size):
        f = W.KERNEL_SPEC.unpack_from(ks, i * W.KERNEL_SPEC.size)
        specs.append(SpkKernelSpec(f[0], f[1], KIND_NAMES.get(f[2], str(f[2])), BACKEND_NAMES.get(f[3], str(f[3])),
                                   f[4], f[5], f[9], f[10], f[6]))
    quant: dict[int, SpkQuant] = {}
    qs = sec(W.SECTION_QUANTIZATION)
    if len(qs) >= W.QUANT_PARAM.size:
        first_off = W.QUANT_PARAM.unpack_from(qs, 0)[4]
        for i in range(first_off // W.QUANT_PARAM.size):
            tid, scheme, axis, nch, off = W.QUANT_PARAM.unpack_from(qs, i * W.QUANT_PARAM.size)
            scales = np.frombuffer(qs, dtype=np.float32, count=nch, offset=off).copy()
            zps = np.frombuffer(qs, dtype=np.int32, count=nch, offset=off + 4 * nch).copy()
            quant[tid] = SpkQuant(tid, scheme, axis, scales, zps)
    plan = []
    ps = sec(W.SECTION_MEMORY_PLAN)
    for i in range(len(ps) // W.MEMORY_PLAN.size):
        plan.append(W.MEMORY_PLAN.unpack_from(ps, i * W.MEMORY_PLAN.size))
    meta = json.loads(sec(W.SECTION_METADATA).decode("utf-8") or "{}")
    prof_raw = sec(W.SECTION_TARGET_PROFILE)
    profile = json.loads(prof_raw.decode("utf-8")) if prof_raw else {}
    return SpkPackage(header, tensors, nodes, specs, quant, sec(W.SECTION_WEIGHTS), meta, profile, plan)


def checksum_ok(src: str | Path | bytes) -> bool:
    data = Path(src).read_bytes() if not isinstance(src, (bytes, bytearray)) else bytes(src)
    pkg_h = W.HEADER.unpack_from(data, 0)
    for i in range(pkg_h[5]):
        kind, _f, off, size, _a, _r = W.SECTION.unpack_from(data, pkg_h[4] + i * W.SECTION.size)
        if kind == W.SECTION_CHECKSUM:
            return struct.unpack_from("<I", data, off)[0] == W.fnv1a32(data[:off])
    return False
