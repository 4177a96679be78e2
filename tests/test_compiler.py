"""Compiler mirror (CPU): byte-identity with the reference compiler, planner
contracts and the cuda_b200 target profile."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import pytest

from spinnv2_b200.compiler import builders, pipeline
from spinnv2_b200.compiler.ir import DTYPE_FP32, ROLE_ACTIVATION, ROLE_INPUT, ROLE_OUTPUT, Graph, Node, Tensor
from spinnv2_b200.compiler.kernel_spec import select_kernel_specs
from spinnv2_b200.compiler.memory_plan import analyze_lifetimes, plan_memory
from spinnv2_b200.compiler.profile import load_target_profile
from spinnv2_b200.spk import checksum_ok, read_spk

GOLDEN = json.loads((Path(__file__).parent / "golden" / "spk_sha256.json").read_text())


@pytest.mark.parametrize("key", sorted(GOLDEN["packages"]))
def test_cpu_package_is_byte_identical_to_reference_compiler(key):
    name, batch = key.rsplit("_b", 1)
    g = pipeline.fuse(builders.build_config(name, int(batch)))
    data = pipeline.package(g, GOLDEN["profile"])
    assert len(data) == GOLDEN["packages"][key]["bytes"]
    assert hashlib.sha256(data).hexdigest() == GOLDEN["packages"][key]["sha256"]
    assert checksum_ok(data)


def _branch_graph() -> Graph:
    # reference tests/compiler/unit/test_memory_plan.py:53-71
    g = Graph(model_name="branch")
    for t in [Tensor(0, "input", DTYPE_FP32, [1, 4], ROLE_INPUT), Tensor(1, "t1", DTYPE_FP32, [1, 4], ROLE_ACTIVATION),
              Tensor(2, "t2", DTYPE_FP32, [1, 4], ROLE_ACTIVATION), Tensor(3, "t3", DTYPE_FP32, [1, 4], ROLE_ACTIVATION),
              Tensor(4, "t4", DTYPE_FP32, [1, 4], ROLE_OUTPUT)]:
        g.add_tensor(t)
    g.inputs, g.outputs = [0], [4]
    for i in range(4):
        g.add_node(Node(i, "Sigmoid", [i], [i + 1]))
    return g


def test_memory_plan_contracts():
    g = _branch_graph()
    life = analyze_lifetimes(g)
    assert life[1] == (0, 1) and life[4] == (3, len(g.nodes) + 1)
    plan = plan_memory(g)
    assert plan.entries[1].offset == plan.entries[3].offset
    assert plan.planned_activation_bytes < plan.naive_activation_bytes
    ext = plan_memory(g, alloc_input=False, alloc_output=False)
    assert ext.entries[0].memory_class == "EXTERNAL" and ext.entries[4].memory_class == "EXTERNAL"
    with pytest.raises(MemoryError):
        plan_memory(g, max_arena_bytes=16)


def test_cuda_profile_specs_have_no_cpu_fallback():
    prof = load_target_profile("cuda_b200")
    g = pipeline.fuse(builders.build_config("lenet5", 1))
    plan = select_kernel_specs(g, prof)
    assert all(s.backend == "delegate" for s in plan.specs)
    assert all(s.fallback_kernel_spec_id == 0xFFFFFFFF for s in plan.specs)
    assert [plan.by_node[n.id].kernel_kind for n in g.nodes if n.op_type == "Conv"] == ["tc_3xtf32"] * 2
    assert plan.scratch_arena_bytes == 0


def test_cuda_plan_keeps_nhwc_safe_aliases_only():
    # LeNet's Flatten of a [1,16,5,5] map: aliased in place for the CPU, not for cuda_b200.
    cpu = read_spk(pipeline.compile_config("lenet5", 1, targets=("cpu_generic_x86",), use_cache=False)["cpu_generic_x86"])
    cuda = read_spk(pipeline.compile_config("lenet5", 1, targets=("cuda_b200",), use_cache=False)["cuda_b200"])
    flat_cpu = next(n for n in cpu.nodes if n.op_type == "Flatten")
    flat_cuda = next(n for n in cuda.nodes if n.op_type == "Flatten")
    assert cpu.tensors[flat_cpu.inputs[0]].data_offset == cpu.tensors[flat_cpu.outputs[0]].data_offset
    assert cuda.tensors[flat_cuda.inputs[0]].data_offset != cuda.tensors[flat_cuda.outputs[0]].data_offset
    assert all(t.data_offset % 256 == 0 for t in cuda.tensors if t.role in (1, 2, 4))
    # YOLO-style at batch 1: no Concat input may live inside its Concat's output.
    y = read_spk(pipeline.compile_config("yolo_style", 1, targets=("cuda_b200",))["cuda_b200"])
    for n in y.nodes:
        if n.op_type == "Concat":
            out = y.tensors[n.outputs[0]]
            for i in n.inputs:
                t = y.tensors[i]
                assert not (out.data_offset <= t.data_offset < out.data_offset + out.size_bytes)


def test_resnet_flops_match_published_counts():
    """2 x MACs of the convs and the FC at 224x224: ResNet-101 v1.5 15.60 and
    ResNet-50 v1.5 8.18 GFLOP per image."""
    assert abs(builders.resnet_gflop_per_image(101) - 15.60) < 0.05
    assert abs(builders.resnet_gflop_per_image(50) - 8.18) < 0.05


def test_unsupported_op_fails_loudly_for_cuda():
    g = Graph(model_name="nms")
    g.add_tensor(Tensor(0, "a", DTYPE_FP32, [2, 2], ROLE_INPUT))
    g.add_tensor(Tensor(1, "b", DTYPE_FP32, [2, 2], ROLE_INPUT))
    g.add_tensor(Tensor(2, "y", DTYPE_FP32, [2, 2], ROLE_OUTPUT))
    g.inputs, g.outputs = [0, 1], [2]
    g.add_node(Node(0, "NonMaxSuppression", [0, 1], [2]))
    with pytest.raises(ValueError):
        select_kernel_specs(g, load_target_profile("cuda_b200"))


def test_cuda_profile_covers_every_runtime_op():
    from spinnv2_b200.compiler.ir import RUNTIME_OPS

    ops = load_target_profile("cuda_b200")["ops"]
    assert RUNTIME_OPS <= set(ops)
    assert not any("ref" in toks for toks in ops.values())  # no CPU fallback spec anywhere
