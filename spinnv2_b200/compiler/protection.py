"""Reliability protection plans: validation and the SPK protection section.

Same format and rules as the reference compiler (reference
compiler/reliability/protection_plan.py:14-131): one 28-byte record per
protected node, `<IIHHffQ` = node id, tensor id, mode code, flags (0), lower
and upper bound (infinite bounds written as -/+FLT_MAX), scratch offset (the
DMR copies start right after the kernel scratch peak; 0 for other modes).
Modes: none 0, range_guard_rerun 1 (rerun the node once when its output has
a non-finite value or one outside [lower, upper]), dmr_compare_rerun 2 (run
twice, compare bytes, a third run votes).  A protected node has exactly one
fp32 output and the record names it.  DMR needs 2 x the output's bytes of
scratch; the package's scratch arena grows by the largest such need.  The
plan JSON (`load_protection_plan`) is the reference's version-1 schema.
"""

from __future__ import annotations

import json
import math
import struct
from dataclasses import dataclass
from pathlib import Path

from .ir import DTYPE_FP32, Graph

RECORD = struct.Struct("<IIHHffQ")
MODE_CODES = {"none": 0, "range_guard_rerun": 1, "dmr_compare_rerun": 2}
FLT_MAX = 3.4028235e38


@dataclass(frozen=True)
class ProtectionEntry:
    node_id: int
    tensor_id: int
    mode: str
    lower_bound: float = -math.inf
    upper_bound: float = math.inf
    compare_atol: float = 0.0
    compare_rtol: float = 0.0


@dataclass(frozen=True)
class ProtectionPlan:
    nodes: tuple[ProtectionEntry, ...]
    version: int = 1
    model_id: str = ""

    def validate(self, graph: Graph) -> "ProtectionPlan":
        seen: set[int] = set()
        for e in self.nodes:
            if e.mode not in MODE_CODES:
                raise ValueError(f"unsupported protection mode: {e.mode}")
            if not 0 <= e.node_id < len(graph.nodes):
                raise ValueError(f"unknown protection node_id: {e.node_id}")
            if e.node_id in seen:
                raise ValueError(f"duplicate protection node_id: {e.node_id}")
            seen.add(e.node_id)
            outs = graph.nodes[e.node_id].outputs
            if len(outs) != 1:
                raise ValueError(f"protected node {e.node_id} must have exactly one output")
            if e.tensor_id != outs[0]:
                raise ValueError(f"tensor {e.tensor_id} is not output of node {e.node_id}")
            if graph.tensors[e.tensor_id].dtype != DTYPE_FP32:
                raise ValueError(f"protected tensor {e.tensor_id} must be fp32")
            if e.mode == "range_guard_rerun" and e.lower_bound > e.upper_bound:
                raise ValueError(f"invalid range for node {e.node_id}")
        return self

    def scratch_bytes(self, graph: Graph) -> int:
        """Extra scratch for the two DMR copies of the largest protected output."""
        return max((2 * graph.tensors[e.tensor_id].size_bytes for e in self.nodes if e.mode == "dmr_compare_rerun"),
                   default=0)

    def section(self, graph: Graph, scratch_offset: int) -> bytes:
        self.validate(graph)
        out = bytearray()
        for e in self.nodes:
            lo = e.lower_bound if math.isfinite(e.lower_bound) else -FLT_MAX
            hi = e.upper_bound if math.isfinite(e.upper_bound) else FLT_MAX
            off = scratch_offset if e.mode == "dmr_compare_rerun" else 0
            out += RECORD.pack(e.node_id, e.tensor_id, MODE_CODES[e.mode], 0, lo, hi, off)
        return bytes(out)


def load_protection_plan(path: str | Path) -> ProtectionPlan:
    """Version-1 plan JSON: {"version": 1, "model_id", "nodes": [{node_id,
    tensor_id, mode, lower_bound?, upper_bound?, compare_atol?, compare_rtol?}]}."""
    return plan_from_dict(json.loads(Path(path).read_text(encoding="utf-8")))


def plan_from_dict(doc: dict) -> ProtectionPlan:
    if int(doc.get("version", 0)) != 1:
        raise ValueError("ProtectionPlan version must be 1")
    entries = tuple(
        ProtectionEntry(int(n["node_id"]), int(n["tensor_id"]), str(n["mode"]),
                        float(n.get("lower_bound", -math.inf)), float(n.get("upper_bound", math.inf)),
                        float(n.get("compare_atol", 0.0)), float(n.get("compare_rtol", 0.0)))
        for n in doc.get("nodes", []))
    return ProtectionPlan(entries, 1, str(doc.get("model_id", "")))
