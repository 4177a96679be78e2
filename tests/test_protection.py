"""Reliability protection plans (range_guard_rerun, dmr_compare_rerun) on the
CUDA target, against the reference SPINNV2 runtime (oracle/_ref).

CPU: the protected LeNet-5 package is byte-identical to the reference
compiler's (tests/golden/spk_sha256.json, "protected"), and plans are
validated as the reference validates them.
GPU: the same graph and plan packaged for cuda_b200 runs under fault events
(single bit flips after a node's n-th execution); reliability statistics must
equal the reference runtime's exactly, outputs match within the fp32
tolerance (max-abs 1e-3, rel 1e-4) and range observations within it too."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import seeded_input

GOLDEN = json.loads((Path(__file__).parent / "golden" / "spk_sha256.json").read_text())
ATOL, RTOL = 1e-3, 1e-4


def _graph():
    from spinnv2_b200.compiler import builders, pipeline

    return pipeline.fuse(builders.build_config("lenet5", 1))


def _plan(graph, tight: bool = False):
    from spinnv2_b200.compiler import builders
    from spinnv2_b200.compiler.protection import plan_from_dict

    entries = builders.lenet5_protection_entries(graph)
    if tight:  # node 0's Relu output exceeds 1.0, so its guard trips on every run
        entries[0] = dict(entries[0], upper_bound=1.0)
    return plan_from_dict({"version": 1, "model_id": "lenet5", "nodes": entries})


def _packages(tight: bool = False):
    import copy

    from spinnv2_b200.compiler import pipeline

    g = _graph()
    plan = _plan(g, tight)
    return {t: pipeline.package(copy.deepcopy(g), t, protection_plan=plan) for t in ("cuda_b200", "cpu_generic_x86")}


def test_protected_package_is_byte_identical_to_reference_compiler():
    from spinnv2_b200.compiler import pipeline

    g = _graph()
    data = pipeline.package(g, GOLDEN["profile"], protection_plan=_plan(g))
    gold = GOLDEN["protected"]["lenet5_b1"]
    assert len(data) == gold["bytes"] and hashlib.sha256(data).hexdigest() == gold["sha256"]


def test_plan_validation_follows_reference_rules():
    from spinnv2_b200.compiler.protection import ProtectionEntry, ProtectionPlan

    g = _graph()
    out0 = g.nodes[0].outputs[0]
    bad = [
        ProtectionPlan((ProtectionEntry(0, out0, "triple_vote"),)),
        ProtectionPlan((ProtectionEntry(99, out0, "dmr_compare_rerun"),)),
        ProtectionPlan((ProtectionEntry(0, out0, "dmr_compare_rerun"),) * 2),
        ProtectionPlan((ProtectionEntry(0, out0 + 1, "dmr_compare_rerun"),)),
        ProtectionPlan((ProtectionEntry(0, out0, "range_guard_rerun", 2.0, 1.0),)),
    ]
    for plan in bad:
        with pytest.raises(ValueError):
            plan.validate(g)
    # DMR scratch: two copies of the largest DMR-protected output.
    assert _plan(g).scratch_bytes(g) == 2 * 16 * 10 * 10 * 4


def _scenarios(x):
    """(name, fault event or None, tight plan): the fault element of node 0 is
    one whose value lies in (0.5, 1), so flipping exponent bit 30 multiplies
    it by 2^128 (still finite) and takes it far outside [0, 60]."""
    from oracle import harness

    spk = _packages()["cuda_b200"]
    _, env = harness.run_spk(spk, [x], keep_all=True)
    g = _graph()
    t0 = g.nodes[0].outputs[0]
    v = env[t0].reshape(-1)
    e0 = int(np.flatnonzero((v > 0.5) & (v < 1.0))[0])
    t2, t9 = g.nodes[2].outputs[0], g.nodes[9].outputs[0]
    ev = lambda node, tid, el, bit, inv: {"node_id": node, "tensor_id": tid, "element_index": el, "bit_index": bit,
                                          "invocation_index": inv, "seed": 0}
    return [
        ("clean", None, False),
        ("range_guard_recovers", ev(0, t0, e0, 30, 1), False),
        ("range_guard_fault_on_rerun", ev(0, t0, e0, 30, 2), True),
        ("dmr_second_copy_faulty", ev(2, t2, 17, 3, 2), False),
        ("dmr_first_copy_faulty", ev(9, t9, 3, 22, 1), False),
        ("dmr_vote_run_faulty", ev(9, t9, 3, 22, 3), False),
        ("unprotected_node_fault", ev(3, g.nodes[3].outputs[0], 5, 29, 1), False),
        ("tight_guard_unrecovered", None, True),
    ]


@pytest.mark.gpu
def test_protected_runs_match_reference_statistics(gpu, tmp_path):
    from oracle import refrt
    from spinnv2_b200.runtime import LIB_PATH, FaultEvent, RuntimeDriver

    x = seeded_input((1, 1, 28, 28), "uniform")
    observed = [0, 5]
    pk = {False: _packages(False), True: _packages(True)}
    for tight in (False, True):
        (tmp_path / f"m{int(tight)}.spk").write_bytes(pk[tight]["cuda_b200"])
    for name, event, tight in _scenarios(x):
        ref = refrt.RefRuntime(pk[tight]["cpu_generic_x86"], [((1, 10), np.float32)])
        try:
            r_out, r_stats, r_obs = ref.run_reliability([x], event, observed)
        finally:
            ref.close()
        with RuntimeDriver(LIB_PATH, tmp_path / f"m{int(tight)}.spk") as drv:
            g_out, g_stats = drv.run(x, FaultEvent(**event) if event else None)
            g_obs = {o["node_id"]: (o["observed_min"], o["observed_max"], o["observations"])
                     for o in drv.range_observations(observed)}
        assert g_stats == r_stats, name
        np.testing.assert_allclose(g_out.reshape(r_out[0].shape), r_out[0], atol=ATOL, rtol=RTOL, err_msg=name)
        assert sorted(g_obs) == sorted(r_obs), name
        for nid in r_obs:
            assert g_obs[nid][2] == r_obs[nid][2], name
            np.testing.assert_allclose(g_obs[nid][:2], r_obs[nid][:2], atol=ATOL, rtol=RTOL, err_msg=name)
