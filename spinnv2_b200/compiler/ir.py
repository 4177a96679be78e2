"""SIR graph model used to build SPK packages for the CUDA target.

Same data model as SPINNV2's compiler IR (reference compiler/ir/graph.py:11-75,
compiler/ir/types.py): tensors and nodes with dense, ordered ids; a tensor has
a dtype, a shape, a role and optional constant bytes; a node has an op type,
input/output tensor ids and an attribute dict.  Graph builders, passes, the
planners and the SPK writer all operate on this model, so a graph built here
can be packaged for the CUDA target and for the reference CPU profiles alike.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import numpy as np

DTYPE_FP32 = "fp32"
DTYPE_INT8 = "int8"
DTYPE_FP16 = "fp16"
DTYPE_INT32 = "int32"  # CUDA target: int32 requantisation bias

ROLE_INPUT = "input"
ROLE_OUTPUT = "output"
ROLE_WEIGHT = "weight"
ROLE_ACTIVATION = "activation"
ROLE_CONSTANT = "constant"

LAYOUT_NCHW = "NCHW"

DTYPE_BYTES = {DTYPE_FP32: 4, DTYPE_INT8: 1, DTYPE_FP16: 2, DTYPE_INT32: 4}
NUMPY_DTYPES = {DTYPE_FP32: np.float32, DTYPE_INT8: np.int8, DTYPE_FP16: np.float16, DTYPE_INT32: np.int32}

# Ops the runtime executes (reference compiler/ir/types.py:15-47).
RUNTIME_OPS = {
    "Add", "AveragePool", "Cast", "Clip", "Concat", "Conv", "Div", "Flatten", "Gather",
    "GatherElements", "Gemm", "GlobalAveragePool", "LeakyRelu", "MatMul", "MaxPool", "Mod",
    "Mul", "ReduceMax", "ReduceMean", "Relu", "Reshape", "Resize", "Sigmoid", "Slice",
    "Softmax", "Split", "Sub", "Tile", "TopK", "Transpose", "Unsqueeze",
}
# Ops that only exist before the passes run.
COMPILER_ONLY_OPS = {"BatchNormalization", "Dropout", "Identity"}


@dataclass
class Tensor:
    id: int
    name: str
    dtype: str
    shape: list[int]
    role: str
    layout: str = LAYOUT_NCHW
    producer: int | None = None
    consumers: list[int] = field(default_factory=list)
    data: bytes | None = None

    @property
    def elem_count(self) -> int:
        n = 1
        for d in self.shape:
            n *= int(d)
        return n

    @property
    def size_bytes(self) -> int:
        if self.dtype not in DTYPE_BYTES:
            raise ValueError(f"unsupported dtype: {self.dtype}")
        return self.elem_count * DTYPE_BYTES[self.dtype]

    def array(self) -> np.ndarray:
        """Constant data as a numpy array of the tensor's dtype and shape."""
        if self.data is None:
            raise ValueError(f"tensor {self.name} has no constant data")
        return np.frombuffer(self.data, dtype=NUMPY_DTYPES[self.dtype]).reshape(self.shape)


@dataclass
class Node:
    id: int
    op_type: str
    inputs: list[int]
    outputs: list[int]
    attrs: dict[str, Any] = field(default_factory=dict)
    execution_index: int = 0


@dataclass
class Graph:
    model_name: str
    tensors: list[Tensor] = field(default_factory=list)
    nodes: list[Node] = field(default_factory=list)
    inputs: list[int] = field(default_factory=list)
    outputs: list[int] = field(default_factory=list)
    metadata: dict[str, Any] = field(default_factory=dict)

    def tensor(self, tensor_id: int) -> Tensor:
        return self.tensors[tensor_id]

    def add_tensor(self, tensor: Tensor) -> None:
        if tensor.id != len(self.tensors):
            raise ValueError("tensor ids must be dense and ordered")
        self.tensors.append(tensor)

    def add_node(self, node: Node) -> None:
        if node.id != len(self.nodes):
            raise ValueError("node ids must be dense and ordered")
        self.nodes.append(node)
        for tid in node.inputs:
            self.tensors[tid].consumers.append(node.id)
        for tid in node.outputs:
            self.tensors[tid].producer = node.id


class GraphBuilder:
    """Convenience layer for writing graphs op by op (model builders)."""

    def __init__(self, name: str) -> None:
        self.graph = Graph(model_name=name)

    def tensor(self, name: str, shape, dtype: str = DTYPE_FP32, role: str = ROLE_ACTIVATION,
               data: np.ndarray | bytes | None = None) -> int:
        tid = len(self.graph.tensors)
        if isinstance(data, np.ndarray):
            data = np.ascontiguousarray(data, dtype=NUMPY_DTYPES[dtype]).tobytes()
        self.graph.add_tensor(Tensor(tid, name, dtype, [int(d) for d in shape], role, data=data))
        return tid

    def weight(self, name: str, value: np.ndarray, dtype: str = DTYPE_FP32) -> int:
        return self.tensor(name, value.shape, dtype, ROLE_WEIGHT, value)

    def input(self, name: str, shape, dtype: str = DTYPE_FP32) -> int:
        tid = self.tensor(name, shape, dtype, ROLE_INPUT)
        self.graph.inputs.append(tid)
        return tid

    def node(self, op: str, inputs: list[int], out_shapes: list, attrs: dict | None = None,
             out_dtype: str = DTYPE_FP32, name: str | None = None) -> list[int]:
        nid = len(self.graph.nodes)
        outs = [self.tensor(f"{name or op.lower()}_{nid}_out{i}", s, out_dtype) for i, s in enumerate(out_shapes)]
        self.graph.add_node(Node(nid, op, list(inputs), outs, dict(attrs or {})))
        return outs

    def op(self, op: str, inputs: list[int], out_shape, attrs: dict | None = None, **kw) -> int:
        return self.node(op, inputs, [out_shape], attrs, **kw)[0]

    def mark_output(self, tid: int) -> None:
        self.graph.tensors[tid].role = ROLE_OUTPUT
        self.graph.outputs.append(tid)

    def shape(self, tid: int) -> list[int]:
        return list(self.graph.tensors[tid].shape)
