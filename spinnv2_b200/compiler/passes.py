"""Graph passes run before kernel selection.

The pass list, order and rewrite rules are SPINNV2's default pipeline
(reference compiler/passes/manager.py:26-53, compiler/passes/transforms.py):
identity/dropout removal, constant folding of Add/Relu/Flatten, Conv+BN
folding, Conv+Relu, Conv+Sigmoid*Mul (SiLU), Add+Relu, Conv+Add (residual as
the conv's fourth input), transpose-pair removal, constant sharing and dead
node elimination.  The fused forms are the epilogue contract of the CUDA
conv kernel (bias, residual, Relu/SiLU), so the rewrites must be the same
ones the CPU runtime sees.  BN folding uses the same fp32 numpy arithmetic
(W' = W * g/sqrt(v+eps), b' = g/sqrt(v+eps) * (b - m) + beta) so both targets
get identical folded weights.

FuseConvAdd runs only for targets whose backends include one with a fused
residual conv; the reference gates it on {simd, cpu} (manager.py:73-90) and
the CUDA target's `delegate` backend is added to that set.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from typing import Callable

import numpy as np

from .ir import (DTYPE_FP32, ROLE_CONSTANT, ROLE_WEIGHT, Graph, Node, Tensor)

FUSED_RESIDUAL_BACKENDS = {"simd", "cpu", "delegate"}


@dataclass
class PassResult:
    name: str
    changed: int
    nodes_before: int
    nodes_after: int
    tensors_before: int
    tensors_after: int


# ---------------------------------------------------------------- helpers

def relink(graph: Graph) -> None:
    """Recompute producer/consumer links and renumber nodes in list order."""
    for t in graph.tensors:
        t.producer = None
        t.consumers = []
    for i, node in enumerate(graph.nodes):
        node.id = i
        node.execution_index = i
        for tid in node.inputs:
            graph.tensors[tid].consumers.append(i)
        for tid in node.outputs:
            graph.tensors[tid].producer = i


def _is_const(graph: Graph, tid: int) -> bool:
    t = graph.tensors[tid]
    return t.data is not None and t.role in (ROLE_WEIGHT, ROLE_CONSTANT)


def _f32(graph: Graph, tid: int) -> np.ndarray:
    t = graph.tensors[tid]
    return np.frombuffer(t.data or b"", dtype=np.float32).copy().reshape(t.shape)


def _store_f32(graph: Graph, tid: int, value: np.ndarray) -> None:
    t = graph.tensors[tid]
    value = np.ascontiguousarray(value, dtype=np.float32)
    t.shape = [int(d) for d in value.shape]
    t.data = value.tobytes()
    t.role = ROLE_WEIGHT


def _new_weight(graph: Graph, name: str, value: np.ndarray) -> int:
    value = np.ascontiguousarray(value, dtype=np.float32)
    tid = len(graph.tensors)
    graph.add_tensor(Tensor(tid, name, DTYPE_FP32, [int(d) for d in value.shape], ROLE_WEIGHT, data=value.tobytes()))
    return tid


def _other_consumers(graph: Graph, tid: int, except_node: int) -> int:
    return sum(1 for n in graph.tensors[tid].consumers if n != except_node)


def _replace_uses(graph: Graph, old: int, new: int) -> None:
    for node in graph.nodes:
        node.inputs = [new if t == old else t for t in node.inputs]
    graph.outputs = [new if t == old else t for t in graph.outputs]


def compact(graph: Graph) -> None:
    """Drop unreferenced tensors and renumber tensors densely."""
    relink(graph)
    used = set(graph.inputs) | set(graph.outputs)
    for node in graph.nodes:
        used.update(node.inputs)
        used.update(node.outputs)
    remap: dict[int, int] = {}
    kept: list[Tensor] = []
    for old, t in enumerate(graph.tensors):
        if old not in used:
            continue
        remap[old] = len(kept)
        kept.append(Tensor(len(kept), t.name, t.dtype, list(t.shape), t.role, layout=t.layout, data=t.data))
    graph.tensors = kept
    graph.inputs = [remap[t] for t in graph.inputs if t in remap]
    graph.outputs = [remap[t] for t in graph.outputs if t in remap]
    for i, node in enumerate(graph.nodes):
        node.id = i
        node.execution_index = i
        node.inputs = [remap[t] for t in node.inputs if t in remap]
        node.outputs = [remap[t] for t in node.outputs if t in remap]
    relink(graph)


def _drop_nodes(graph: Graph, doomed: set[int]) -> None:
    if doomed:
        graph.nodes = [n for n in graph.nodes if n.id not in doomed]
        compact(graph)


def topo_sort(graph: Graph) -> None:
    """Kahn's algorithm over producer edges, FIFO among ready nodes."""
    relink(graph)
    producer = {}
    for i, node in enumerate(graph.nodes):
        for t in node.outputs:
            producer[t] = i
    succ: list[list[int]] = [[] for _ in graph.nodes]
    indeg = [0] * len(graph.nodes)
    for i, node in enumerate(graph.nodes):
        for t in node.inputs:
            p = producer.get(t)
            if p is not None and p != i:
                succ[p].append(i)
                indeg[i] += 1
    ready = deque(i for i in range(len(graph.nodes)) if indeg[i] == 0)
    order = []
    while ready:
        u = ready.popleft()
        order.append(u)
        for v in succ[u]:
            indeg[v] -= 1
            if indeg[v] == 0:
                ready.append(v)
    graph.nodes = [graph.nodes[i] for i in order]


# ---------------------------------------------------------------- passes

def eliminate_identity_dropout(graph: Graph) -> int:
    changed = 0
    keep: list[Node] = []
    for node in graph.nodes:
        if node.op_type in ("Identity", "Dropout") and node.inputs and node.outputs:
            if not any(t in graph.outputs for t in node.outputs):
                _replace_uses(graph, node.outputs[0], node.inputs[0])
                changed += 1
                continue
        keep.append(node)
    graph.nodes = keep
    compact(graph)
    return changed


def constant_fold(graph: Graph) -> int:
    changed = 0
    keep: list[Node] = []
    for node in graph.nodes:
        foldable = (node.op_type in ("Add", "Relu", "Flatten")
                    and not any(t in graph.outputs for t in node.outputs)
                    and all(_is_const(graph, t) for t in node.inputs))
        value = _fold_value(graph, node) if foldable else None
        if value is not None:
            out = graph.tensors[node.outputs[0]]
            out.data = np.ascontiguousarray(value, dtype=np.float32).tobytes()
            out.shape = [int(d) for d in value.shape]
            out.role = ROLE_WEIGHT
            changed += 1
            continue
        keep.append(node)
    graph.nodes = keep
    compact(graph)
    return changed


def _fold_value(graph: Graph, node: Node) -> np.ndarray | None:
    vals = [_f32(graph, t) for t in node.inputs]
    if node.op_type == "Add":
        return vals[0] + vals[1]
    if node.op_type == "Relu":
        return np.maximum(vals[0], 0.0)
    if node.op_type == "Flatten":
        axis = int(node.attrs.get("axis", 1))
        s = vals[0].shape
        return vals[0].reshape(int(np.prod(s[:axis])), int(np.prod(s[axis:])))
    return None


def fuse_conv_batchnorm(graph: Graph) -> int:
    relink(graph)
    doomed: set[int] = set()
    for bn in list(graph.nodes):
        if bn.op_type != "BatchNormalization" or len(bn.inputs) < 5:
            continue
        src = bn.inputs[0]
        pid = graph.tensors[src].producer
        if pid is None or graph.nodes[pid].op_type != "Conv":
            continue
        conv = graph.nodes[pid]
        if _other_consumers(graph, src, bn.id) != 0:
            continue
        if not all(_is_const(graph, t) for t in bn.inputs[1:5]):
            continue
        w = _f32(graph, conv.inputs[1])
        if w.ndim != 4:
            continue
        oc = w.shape[0]
        gamma, beta, mean, var = (_f32(graph, t).reshape(oc) for t in bn.inputs[1:5])
        eps = float(bn.attrs.get("epsilon", 1e-5))
        factor = gamma / np.sqrt(var + eps)
        if len(conv.inputs) >= 3 and _is_const(graph, conv.inputs[2]):
            b_id = conv.inputs[2]
            b = _f32(graph, b_id).reshape(oc)
        else:
            b = np.zeros((oc,), dtype=np.float32)
            b_id = _new_weight(graph, f"{graph.tensors[conv.inputs[1]].name}_bn_bias", b)
            conv.inputs.append(b_id)
        _store_f32(graph, conv.inputs[1], w * factor.reshape(oc, 1, 1, 1))
        _store_f32(graph, b_id, factor * (b - mean) + beta)
        conv.outputs[0] = bn.outputs[0]
        graph.tensors[bn.outputs[0]].producer = conv.id
        doomed.add(bn.id)
    _drop_nodes(graph, doomed)
    return len(doomed)


def fuse_conv_relu(graph: Graph) -> int:
    relink(graph)
    doomed: set[int] = set()
    for relu in list(graph.nodes):
        if relu.op_type != "Relu" or not relu.inputs or not relu.outputs:
            continue
        src = relu.inputs[0]
        pid = graph.tensors[src].producer
        if pid is None or graph.nodes[pid].op_type != "Conv":
            continue
        if _other_consumers(graph, src, relu.id) != 0:
            continue
        conv = graph.nodes[pid]
        conv.attrs["fused_activation"] = "Relu"
        conv.outputs[0] = relu.outputs[0]
        doomed.add(relu.id)
    _drop_nodes(graph, doomed)
    return len(doomed)


def fuse_conv_silu(graph: Graph) -> int:
    relink(graph)
    doomed: set[int] = set()
    for conv in list(graph.nodes):
        if conv.op_type != "Conv" or not conv.outputs:
            continue
        out = conv.outputs[0]
        users = [graph.nodes[n] for n in graph.tensors[out].consumers]
        if len(users) != 2:
            continue
        sig = next((n for n in users if n.op_type == "Sigmoid"), None)
        mul = next((n for n in users if n.op_type == "Mul"), None)
        if sig is None or mul is None or not sig.outputs or not mul.outputs:
            continue
        sig_out = sig.outputs[0]
        if _other_consumers(graph, sig_out, mul.id) != 0:
            continue
        if not {out, sig_out} <= set(mul.inputs):
            continue
        conv.attrs["fused_activation"] = "Silu"
        conv.outputs[0] = mul.outputs[0]
        graph.tensors[mul.outputs[0]].producer = conv.id
        doomed.update({sig.id, mul.id})
    _drop_nodes(graph, doomed)
    return len(doomed) // 2


def fuse_add_relu(graph: Graph) -> int:
    relink(graph)
    doomed: set[int] = set()
    for relu in list(graph.nodes):
        if relu.op_type != "Relu" or not relu.inputs or not relu.outputs:
            continue
        src = relu.inputs[0]
        pid = graph.tensors[src].producer
        if pid is None or graph.nodes[pid].op_type != "Add":
            continue
        if _other_consumers(graph, src, relu.id) != 0:
            continue
        add = graph.nodes[pid]
        add.attrs["fused_activation"] = "Relu"
        add.outputs[0] = relu.outputs[0]
        graph.tensors[relu.outputs[0]].producer = add.id
        doomed.add(relu.id)
    _drop_nodes(graph, doomed)
    return len(doomed)


def fuse_conv_add(graph: Graph) -> int:
    """Conv(...) -> t; Add(t, r) -> y  becomes  Conv(..., bias, r) -> y."""
    relink(graph)
    doomed: set[int] = set()
    for add in list(graph.nodes):
        if add.op_type != "Add" or len(add.inputs) != 2 or not add.outputs:
            continue
        for side in (0, 1):
            src, residual = add.inputs[side], add.inputs[1 - side]
            pid = graph.tensors[src].producer
            if pid is None or graph.nodes[pid].op_type != "Conv":
                continue
            conv = graph.nodes[pid]
            if _other_consumers(graph, src, add.id) != 0 or conv.attrs.get("fused_activation"):
                continue
            if len(conv.inputs) < 3:
                oc = graph.tensors[conv.inputs[1]].shape[0]
                conv.inputs.append(_new_weight(graph, f"{graph.tensors[conv.inputs[1]].name}_zero_bias",
                                               np.zeros((oc,), dtype=np.float32)))
            conv.inputs.append(residual)
            if add.attrs.get("fused_activation"):
                conv.attrs["fused_activation"] = add.attrs["fused_activation"]
            conv.outputs[0] = add.outputs[0]
            graph.tensors[add.outputs[0]].producer = conv.id
            doomed.add(add.id)
            break
    if doomed:
        graph.nodes = [n for n in graph.nodes if n.id not in doomed]
        topo_sort(graph)
        compact(graph)
    return len(doomed)


def eliminate_noop_transpose(graph: Graph) -> int:
    relink(graph)
    doomed: set[int] = set()
    changed = 0
    for second in list(graph.nodes):
        if second.op_type != "Transpose" or second.id in doomed:
            continue
        mid = second.inputs[0]
        pid = graph.tensors[mid].producer
        if pid is None:
            continue
        first = graph.nodes[pid]
        if first.op_type != "Transpose" or first.id in doomed:
            continue
        if _other_consumers(graph, mid, second.id) != 0:
            continue
        p1, p2 = first.attrs.get("perm", []), second.attrs.get("perm", [])
        if not p1 or not p2 or len(p1) != len(p2):
            continue
        if [p1[p] for p in p2] != list(range(len(p1))):
            continue
        _replace_uses(graph, second.outputs[0], first.inputs[0])
        doomed.update({first.id, second.id})
        changed += 2
    _drop_nodes(graph, doomed)
    return changed


def share_constants(graph: Graph) -> int:
    first_seen: dict[tuple, int] = {}
    redirect: dict[int, int] = {}
    for t in graph.tensors:
        if t.role not in (ROLE_WEIGHT, ROLE_CONSTANT) or t.data is None:
            continue
        key = (tuple(t.shape), t.data)
        if key in first_seen:
            redirect[t.id] = first_seen[key]
        else:
            first_seen[key] = t.id
    for old, new in redirect.items():
        _replace_uses(graph, old, new)
    if redirect:
        compact(graph)
    return len(redirect)


def eliminate_dead(graph: Graph) -> int:
    relink(graph)
    live_nodes: set[int] = set()
    live_tensors = set(graph.outputs)
    work = list(graph.outputs)
    while work:
        tid = work.pop()
        p = graph.tensors[tid].producer
        if p is None or p in live_nodes:
            continue
        live_nodes.add(p)
        for t in graph.nodes[p].inputs:
            if t not in live_tensors:
                live_tensors.add(t)
                work.append(t)
    before = len(graph.nodes)
    graph.nodes = [n for n in graph.nodes if n.id in live_nodes]
    compact(graph)
    return before - len(graph.nodes)


PASSES: dict[str, Callable[[Graph], int]] = {
    "EliminateIdentityDropout": eliminate_identity_dropout,
    "ConstantFold": constant_fold,
    "FuseConvBatchNorm": fuse_conv_batchnorm,
    "FuseConvRelu": fuse_conv_relu,
    "FuseConvSilu": fuse_conv_silu,
    "FuseAddRelu": fuse_add_relu,
    "FuseConvAdd": fuse_conv_add,
    "EliminateNoopTranspose": eliminate_noop_transpose,
    "ShareConstants": share_constants,
    "EliminateDead": eliminate_dead,
}

DEFAULT_PIPELINE = list(PASSES)

# Passes that need a backend able to run their fused form.
PASS_BACKENDS = {"FuseConvAdd": FUSED_RESIDUAL_BACKENDS}


def pipeline_for_target(profile: dict | None = None, pipeline: list[str] | None = None) -> list[str]:
    names = list(pipeline or DEFAULT_PIPELINE)
    if profile is None:
        return names
    backends = set(profile.get("backends", []))
    return [n for n in names if n not in PASS_BACKENDS or PASS_BACKENDS[n] & backends]


def run_pass_pipeline(graph: Graph, *, pipeline: list[str] | None = None, profile: dict | None = None,
                      enabled: bool = True) -> list[PassResult]:
    if not enabled:
        graph.metadata["pass_stats"] = []
        return []
    results = []
    for name in pipeline_for_target(profile, pipeline):
        fn = PASSES[name]
        nb, tb = len(graph.nodes), len(graph.tensors)
        changed = fn(graph)
        relink(graph)
        results.append(PassResult(name, changed, nb, len(graph.nodes), tb, len(graph.tensors)))
    graph.metadata["pass_stats"] = [r.__dict__ for r in results]
    return results
