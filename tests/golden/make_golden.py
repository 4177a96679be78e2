"""Regenerate the compiler golden fixtures from the REFERENCE compiler.

Run where the reference tree is available, giving its root as the argument
or in SPKV2_REFERENCE_ROOT:
    python tests/golden/make_golden.py <reference_root>
For each config it builds the same SIR graph, runs the reference compiler's
pass pipeline, KernelSpec planner, memory planner and SPK writer with the
x86 CPU profile, and records the SHA-256 of the package.  The tests check
that spinnv2_b200's compiler produces byte-identical packages.  It also
records the reference weight quantiser's output on the ResNet-50 graph.
"""

from __future__ import annotations

import copy
import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPKV2_REFERENCE_ROOT")
if not _root:
    sys.exit("usage: make_golden.py <reference_root>  (or set SPKV2_REFERENCE_ROOT)")
REF = Path(_root)
sys.path.insert(0, str(REF))

import numpy as np  # noqa: E402

from compiler.ir import graph as rg  # noqa: E402  (reference compiler)
from compiler.packager.spk_writer import write_spk as ref_write  # noqa: E402
from compiler.passes.manager import run_pass_pipeline as ref_passes  # noqa: E402
from compiler.planner.kernel_spec import select_kernel_specs as ref_specs  # noqa: E402
from compiler.planner.memory_plan import plan_memory as ref_plan  # noqa: E402
from compiler.quantization.quantize_weights import quantize_conv_weights as ref_quantize  # noqa: E402

from spinnv2_b200.compiler import builders  # noqa: E402
from spinnv2_b200.compiler.profile import load_target_profile  # noqa: E402

CONFIGS = [("lenet5", 1), ("yolo_style", 1), ("resnet50", 1), ("resnet101", 1)] + \
          [(c, 1) for c in builders.SWEEP_CASES] + [("conv3x3_64_56", 2), ("gemm_2048_1000", 3)]


def to_reference_graph(g):
    r = rg.Graph(model_name=g.model_name)
    for t in g.tensors:
        r.add_tensor(rg.Tensor(t.id, t.name, t.dtype, list(t.shape), t.role, data=t.data))
    r.inputs, r.outputs = list(g.inputs), list(g.outputs)
    for n in g.nodes:
        r.add_node(rg.Node(n.id, n.op_type, list(n.inputs), list(n.outputs), copy.deepcopy(n.attrs)))
    return r


def main():
    prof = load_target_profile("cpu_generic_x86")
    out = {"profile": "cpu_generic_x86", "packages": {}}
    for name, batch in CONFIGS:
        rgraph = to_reference_graph(builders.build_config(name, batch))
        ref_passes(rgraph, profile=prof)
        with tempfile.TemporaryDirectory() as d:
            ref_write(rgraph, d + "/m.spk", prof, kernel_plan=ref_specs(rgraph, prof),
                      memory_plan=ref_plan(rgraph, max_arena_bytes=prof["memory"]["activation_arena_max"]))
            data = Path(d, "m.spk").read_bytes()
        out["packages"][f"{name}_b{batch}"] = {"sha256": hashlib.sha256(data).hexdigest(), "bytes": len(data)}
        print(name, batch, len(data), flush=True)
    # LeNet-5 with the protection plan of builders.LENET5_PROTECTION, through
    # the reference protection-plan encoder and writer.
    from compiler.reliability.protection_plan import ProtectionEntry as RefEntry  # noqa: E402
    from compiler.reliability.protection_plan import ProtectionPlan as RefPlan  # noqa: E402

    rgraph = to_reference_graph(builders.build_config("lenet5", 1))
    ref_passes(rgraph, profile=prof)
    entries = tuple(RefEntry(**e) for e in builders.lenet5_protection_entries(rgraph))
    with tempfile.TemporaryDirectory() as d:
        ref_write(rgraph, d + "/m.spk", prof, kernel_plan=ref_specs(rgraph, prof),
                  memory_plan=ref_plan(rgraph, max_arena_bytes=prof["memory"]["activation_arena_max"]),
                  protection_plan=RefPlan(version=1, model_id="lenet5", nodes=entries))
        data = Path(d, "m.spk").read_bytes()
    out["protected"] = {"lenet5_b1": {"sha256": hashlib.sha256(data).hexdigest(), "bytes": len(data)}}
    # Reference weight quantiser on the fused ResNet-50 graph.
    rgraph = to_reference_graph(builders.build_config("resnet50", 1))
    ref_passes(rgraph, profile=prof)
    qps = ref_quantize(rgraph)
    h = hashlib.sha256()
    for qp in qps:
        h.update(rgraph.tensors[qp.tensor_id].data)
        h.update(np.asarray(qp.scales, dtype=np.float64).tobytes())
    out["resnet50_weight_quant"] = {"tensors": len(qps), "sha256": h.hexdigest()}
    Path(__file__).with_name("spk_sha256.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
