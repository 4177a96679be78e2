"""Static activation-arena planning.

Algorithm (same steps as reference compiler/planner/memory_plan.py:46-379,
since the arena offsets written into the SPK must be a valid plan for both
runtimes): lifetimes = [producer index, last consumer index] with graph
outputs live to the end; tensors are placed in order of first use into a
best-fit free list (smallest block that fits, split and coalesced) with
`alignment`-byte rounding, growing the arena when nothing fits; in-place
aliases for Reshape/Flatten/Unsqueeze/Cast and single-consumer Relu; Concat
inputs become sub-regions of the Concat output when the outer extent is 1.

CUDA-target options (profile["memory_plan"]):
  concat_alias=false           Concat sub-region aliases are only contiguous
                               in NCHW; with NHWC activations Concat is a
                               kernel that writes channel-interleaved rows.
  layout_changing_alias=false  no in-place alias between a rank-4 tensor with
                               C>1 and H*W>1 and a view of another shape
                               (e.g. Flatten), whose element order differs
                               between NHWC storage and the logical order.
The profile's `alignment` (256 for cuda_b200) rounds every tensor so each
starts on a 256-byte boundary (TMA/vector friendly); the reference uses 16.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

from .ir import ROLE_CONSTANT, ROLE_INPUT, ROLE_OUTPUT, ROLE_WEIGHT, Graph, Tensor

DEFAULT_ALIGNMENT = 16
GRAPH_END_EXTRA = 1
SHAPE_ONLY_OPS = {"Reshape", "Flatten", "Unsqueeze", "Cast"}
INPLACE_ELEMENTWISE_OPS = {"Relu"}


@dataclass
class MemoryPlanEntry:
    tensor_id: int
    name: str
    size: int
    aligned_size: int
    first_use: int
    last_use: int
    offset: int
    memory_class: str


@dataclass
class MemoryPlan:
    entries: dict[int, MemoryPlanEntry]
    naive_activation_bytes: int
    planned_activation_bytes: int
    alloc_input: bool = True
    alloc_output: bool = True

    @property
    def memory_reduction_ratio(self) -> float:
        if self.naive_activation_bytes == 0:
            return 0.0
        return 1.0 - self.planned_activation_bytes / self.naive_activation_bytes


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def analyze_lifetimes(graph: Graph) -> dict[int, tuple[int, int]]:
    end = len(graph.nodes) + GRAPH_END_EXTRA
    outs = set(graph.outputs)
    life: dict[int, tuple[int, int]] = {}
    for t in graph.tensors:
        if t.role == ROLE_WEIGHT:
            life[t.id] = (-1, end)
            continue
        first = 0 if t.producer is None else t.producer
        if t.id in outs:
            last = end
        elif t.consumers:
            last = max(t.consumers)
        else:
            last = first
        life[t.id] = (first, last)
    return life


def _allocated(t: Tensor, alloc_input: bool, alloc_output: bool) -> bool:
    if t.role in (ROLE_WEIGHT, ROLE_CONSTANT):
        return False
    if t.role == ROLE_INPUT and not alloc_input:
        return False
    if t.role == ROLE_OUTPUT and not alloc_output:
        return False
    return t.size_bytes > 0


def _memory_class(t: Tensor, alloc_input: bool, alloc_output: bool) -> str:
    if t.role in (ROLE_WEIGHT, ROLE_CONSTANT):
        return "WEIGHT"
    if t.role == ROLE_INPUT:
        return "INPUT" if alloc_input else "EXTERNAL"
    if t.role == ROLE_OUTPUT:
        return "OUTPUT" if alloc_output else "EXTERNAL"
    return "ACTIVATION_ARENA"


def _layout_sensitive(t: Tensor) -> bool:
    return len(t.shape) == 4 and t.shape[1] > 1 and t.shape[2] * t.shape[3] > 1


def _inplace_aliases(graph: Graph, ai: bool, ao: bool, allow_layout_change: bool) -> dict[int, int]:
    alias: dict[int, int] = {}
    outs, ins = set(graph.outputs), set(graph.inputs)
    for node in graph.nodes:
        shape_only = node.op_type in SHAPE_ONLY_OPS
        elementwise = node.op_type in INPLACE_ELEMENTWISE_OPS
        if not (shape_only or elementwise) or not node.inputs or not node.outputs:
            continue
        src, dst = node.inputs[0], node.outputs[0]
        ts, td = graph.tensors[src], graph.tensors[dst]
        if ts.size_bytes != td.size_bytes:
            continue
        if not _allocated(td, ai, ao) or not _allocated(ts, ai, ao):
            continue
        if dst in outs and src in ins:
            continue
        if elementwise and len(ts.consumers) > 1:
            continue
        if (not allow_layout_change and shape_only and ts.shape != td.shape
                and (_layout_sensitive(ts) or _layout_sensitive(td))):
            continue
        root = alias.get(src, src)
        if elementwise and root in ins:
            continue
        alias[dst] = root
    return alias


def _concat_aliases(graph: Graph, ai: bool, ao: bool) -> dict[int, tuple[int, int]]:
    alias: dict[int, tuple[int, int]] = {}
    ins = set(graph.inputs)
    taken: set[int] = set()
    for node in graph.nodes:
        if node.op_type != "Concat" or len(node.inputs) < 2 or not node.outputs:
            continue
        out = graph.tensors[node.outputs[0]]
        if not _allocated(out, ai, ao):
            continue
        rank = len(out.shape)
        axis = int(node.attrs.get("axis", 0))
        axis = axis + rank if axis < 0 else axis
        if axis < 0 or axis >= rank:
            continue
        outer = 1
        for d in out.shape[:axis]:
            outer *= d
        if outer != 1:
            continue
        inner = 1
        for d in out.shape[axis + 1:]:
            inner *= d
        placed: list[tuple[int, int]] = []
        cursor = 0
        ok = True
        for tid in node.inputs:
            t = graph.tensors[tid]
            byte_off = cursor * inner * 4
            if (not _allocated(t, ai, ao) or tid in ins or tid in taken or byte_off % DEFAULT_ALIGNMENT != 0):
                ok = False
                break
            placed.append((tid, byte_off))
            cursor += t.shape[axis]
        if not ok:
            continue
        for tid, off in placed:
            alias[tid] = (out.id, off)
            taken.add(tid)
    return alias


def _best_fit(free: list[tuple[int, int]], size: int) -> int | None:
    best = None
    for i, (_, bsize) in enumerate(free):
        if bsize >= size and (best is None or bsize < free[best][1]):
            best = i
    if best is None:
        return None
    off, bsize = free.pop(best)
    if bsize > size:
        _release(free, off + size, bsize - size)
    return off


def _release(free: list[tuple[int, int]], off: int, size: int) -> None:
    if size <= 0:
        return
    free.append((off, size))
    free.sort()
    merged: list[tuple[int, int]] = []
    for o, s in free:
        if merged and merged[-1][0] + merged[-1][1] == o:
            merged[-1] = (merged[-1][0], merged[-1][1] + s)
        else:
            merged.append((o, s))
    free[:] = merged


def plan_memory(graph: Graph, *, max_arena_bytes: int = 0, alloc_input: bool = True, alloc_output: bool = True,
                alignment: int = DEFAULT_ALIGNMENT, concat_alias: bool = True,
                layout_changing_alias: bool = True) -> MemoryPlan:
    ai, ao = alloc_input, alloc_output
    life = analyze_lifetimes(graph)
    inplace = _inplace_aliases(graph, ai, ao, layout_changing_alias)
    concat = _concat_aliases(graph, ai, ao) if concat_alias else {}
    for a, src in inplace.items():
        life[src] = (min(life[src][0], life[a][0]), max(life[src][1], life[a][1]))
    for a, (parent, _) in concat.items():
        life[parent] = (min(life[parent][0], life[a][0]), max(life[parent][1], life[a][1]))

    planned = [t for t in graph.tensors if _allocated(t, ai, ao) and t.id not in inplace and t.id not in concat]
    naive = sum(_align(t.size_bytes, alignment) for t in planned)
    entries: dict[int, MemoryPlanEntry] = {}
    free: list[tuple[int, int]] = []
    live: list[tuple[int, int, int]] = []
    peak = 0
    for t in sorted(planned, key=lambda t: (life[t.id][0], t.id)):
        first = life[t.id][0]
        keep = []
        for tid, off, size in live:
            if life[tid][1] < first:
                _release(free, off, size)
            else:
                keep.append((tid, off, size))
        live = keep
        size = _align(t.size_bytes, alignment)
        off = _best_fit(free, size)
        if off is None:
            off = peak
            peak += size
        live.append((t.id, off, size))
        entries[t.id] = MemoryPlanEntry(t.id, t.name, t.size_bytes, size, life[t.id][0], life[t.id][1], off,
                                        _memory_class(t, ai, ao))
    for t in graph.tensors:
        if t.id in entries:
            continue
        first, last = life.get(t.id, (-1, -1))
        if t.id in inplace:
            off = entries[inplace[t.id]].offset
        elif t.id in concat:
            parent, byte_off = concat[t.id]
            off = entries[parent].offset + byte_off
        else:
            off = 0
        entries[t.id] = MemoryPlanEntry(t.id, t.name, t.size_bytes, _align(t.size_bytes, alignment), first, last, off,
                                        _memory_class(t, ai, ao))
    if max_arena_bytes > 0 and peak > max_arena_bytes:
        raise MemoryError(f"planned activation arena {peak} exceeds target limit {max_arena_bytes}")
    return MemoryPlan(entries, naive, peak, ai, ao)


def plan_for_profile(graph: Graph, profile: dict, **kw) -> MemoryPlan:
    opts = profile.get("memory_plan", {})
    return plan_memory(graph, max_arena_bytes=int(profile["memory"]["activation_arena_max"]),
                       alignment=int(profile.get("alignment", DEFAULT_ALIGNMENT)) if "memory_plan" in profile
                       else DEFAULT_ALIGNMENT,
                       concat_alias=bool(opts.get("concat_alias", True)),
                       layout_changing_alias=bool(opts.get("layout_changing_alias", True)), **kw)


def write_memory_plan_csv(plan: MemoryPlan, path: str | Path) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    rows = ["tensor_id,name,size,aligned_size,first_use,last_use,offset,memory_class"]
    for tid in sorted(plan.entries):
        e = plan.entries[tid]
        rows.append(f"{e.tensor_id},{e.name},{e.size},{e.aligned_size},{e.first_use},{e.last_use},{e.offset},"
                    f"{e.memory_class}")
    path.write_text("\n".join(rows) + "\n", encoding="utf-8")
