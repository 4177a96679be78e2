"""GPU parity on the configurations bench.py measures, at their batch sizes.

- ResNet-101 fp32 (3xTF32) at batch 64 and 256: the graph-replayed plan
  (eager run, capture, replay) with the same tiles and stream-K splits as the
  benchmark, final logits checked ELEMENT-WISE against the reference CPU
  runtime (oracle/_ref) with the fp32 tolerance of the north star,
  np.testing.assert_allclose(atol=1e-3, rtol=1e-4).  The logits are an extra
  graph output of the same fused graph, so the reference computes them too.
- INT8 ResNet-50 at batch 256, node by node on the GPU: every int8 conv
  output, MaxPool and ReduceMean bit-exact against the oracle run on the
  GPU's own inputs to that node, for images 0, 1, 254 and 255 (the first and
  the last M tiles of every layer).
- The YOLOv10n-style detector at batch 1 and 64: top-300 scores within tolerance;
  where a TopK index differs from the reference's, the reference's score of
  the GPU's anchor must tie (within tolerance) with the reference's score at
  that rank, and every GPU box must equal the reference's box of the anchor
  the GPU chose.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import compile_with_outputs, gemm_output, reference_outputs, seeded_input

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4


def _report(name: str, got: np.ndarray, want: np.ndarray) -> None:
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    i = int(np.argmax(err))
    rel = err / np.maximum(np.abs(want.astype(np.float64)), 1e-30)
    used = err / (ATOL + RTOL * np.abs(want.astype(np.float64)))
    print(f"{name}: worst abs {err.flat[i]:.3e} at ref {want.flat[i]:.4g}; worst rel {rel.max():.3e}; "
          f"|ref| max {np.abs(want).max():.4g}; allowed at worst abs {ATOL + RTOL * abs(want.flat[i]):.3e}; "
          f"largest share of the tolerance used {used.max():.3f}")


@pytest.mark.parametrize("batch", [64, 256])
def test_resnet101_bench_batch_graph_replay_logits_elementwise(gpu, batch):
    from spinnv2_b200.runtime import Runtime

    spk = compile_with_outputs("resnet101", batch, gemm_output)
    x = seeded_input((batch, 3, 224, 224), seed=17)
    ref_probs, ref_logits = reference_outputs(spk["cpu_generic_x86"], [x])
    with Runtime(spk["cuda_b200"], device=0, graph=True) as rt:
        runs = [rt.run(x) for _ in range(3)]  # eager, capture, replay
        convs = [n.id for n in rt.package.nodes if n.op_type == "Conv"]
        variants = {rt.node_variant(i) for i in convs}
    probs, logits = runs[-1]
    _report(f"resnet101 bs{batch} logits", logits, ref_logits)
    assert any("_sk_" in v for v in variants), variants  # the benchmark's stream-K tails are in the plan
    assert 1.0 < float(np.abs(ref_logits).max()) < 1e3  # logits of a sane scale (not cancellation noise)
    np.testing.assert_allclose(logits, ref_logits, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(probs, ref_probs, atol=ATOL, rtol=RTOL)
    np.testing.assert_array_equal(runs[2][1], runs[1][1])  # replay repeats the captured run bit for bit


def test_int8_resnet50_bs256_every_node_on_edge_images(gpu):
    from oracle import harness
    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import Runtime
    from spinnv2_b200.spk import read_spk

    spk = pipeline.compile_config("resnet50", 256, targets=("cuda_b200",), int8=True)["cuda_b200"]
    pkg = read_spk(spk)
    pick = np.array([0, 1, 254, 255])
    # The oracle runs each node on the 4 picked images: the same network
    # packaged at batch 4 (same weights, same calibration, same ids).
    pkg4 = read_spk(pipeline.compile_config("resnet50", len(pick), targets=("cuda_b200",), int8=True)["cuda_b200"])
    assert [n.op_type for n in pkg4.nodes] == [n.op_type for n in pkg.nodes]
    for t, q in pkg.quant.items():
        np.testing.assert_array_equal(np.asarray(pkg4.quant[t].scales), np.asarray(q.scales), err_msg=str(t))
    x = seeded_input((256, 3, 224, 224), seed=23)
    convs = [n for n in pkg.nodes if n.op_type == "Conv"]
    with Runtime(spk, device=0) as rt:
        rt.run(x)
        rt.set_input(0, x)
        gpu_t = {pkg.inputs[0].id: x[pick]}
        for n in pkg.nodes:  # one node at a time: each output read right after its node
            rt.run_nodes(n.id, n.id + 1)
            for t in n.outputs:
                gpu_t[t] = rt.read_tensor(t)[pick]
        variants = {n.id: rt.node_variant(n.id) for n in convs}
    assert all(variants[n.id].startswith("tc_int8") for n in convs[1:]), variants
    checked = 0
    for n in pkg.nodes:
        env = {t: gpu_t[t] for t in n.inputs if t in gpu_t}
        want = harness.run_node(pkg4, n, env)[0]
        got = gpu_t[n.outputs[0]]
        if n.id == convs[0].id:
            # fp32-math stem with an int8 output: one code where fp32
            # summation order crosses a rounding boundary.
            diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
            assert diff.max() <= 1 and (diff > 0).mean() < 1e-3, (diff.max(), (diff > 0).mean())
        elif got.dtype == np.int8 or n.op_type == "ReduceMean":
            np.testing.assert_array_equal(got, want, err_msg=f"node {n.id} {n.op_type} {variants.get(n.id, '')}")
            checked += 1
        else:
            np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL, err_msg=f"node {n.id} {n.op_type}")
    assert checked >= len(convs) - 1


def _yolo_pick(graph) -> list[int]:
    """Per-anchor best class score (ReduceMax output) and per-anchor boxes
    (the Transpose output that GatherElements indexes)."""
    return [n.outputs[0] for n in graph.nodes if n.op_type in ("ReduceMax", "Transpose")]


@pytest.mark.parametrize("batch", [1, 64])
def test_yolo_style_topk_disagreements_are_ties(gpu, batch):
    from spinnv2_b200.runtime import Runtime

    spk = compile_with_outputs("yolo_style", batch, _yolo_pick)
    x = seeded_input((batch, 3, 640, 640), "uniform", seed=29)
    ref_vals, ref_boxes, ref_best, ref_anchor_boxes = reference_outputs(spk["cpu_generic_x86"], [x])
    with Runtime(spk["cuda_b200"], device=0, graph=True) as rt:
        rt.run(x)
        vals, boxes, best, _ = rt.run(x)
        topk = next(n for n in rt.package.nodes if n.op_type == "TopK")
        idx = rt.read_tensor(topk.outputs[1]).astype(np.int64)
    _report(f"yolo bs{batch} top-300 scores", vals, ref_vals)
    np.testing.assert_allclose(best, ref_best, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(vals, ref_vals, atol=ATOL, rtol=RTOL)
    # The GPU's anchor at every rank scores (by the reference) the same as
    # the reference's anchor at that rank, within tolerance: disagreements
    # are ties, not selection errors.
    ref_score_of_gpu_pick = np.take_along_axis(ref_best, idx, axis=1)
    np.testing.assert_allclose(ref_score_of_gpu_pick, ref_vals, atol=ATOL, rtol=RTOL)
    assert all(len(set(row)) == row.size for row in idx)  # no anchor picked twice
    # Boxes: the GPU's box of each chosen anchor equals the reference's box of that anchor.
    want_boxes = np.take_along_axis(ref_anchor_boxes, idx[:, :, None].repeat(4, axis=2), axis=1)
    np.testing.assert_allclose(boxes, want_boxes, atol=ATOL, rtol=RTOL)
    same = (idx == np.rint(reference_indices(ref_best, ref_vals)).astype(np.int64)).mean()
    print(f"yolo bs{batch}: {100 * same:.2f} % of TopK indices identical to the reference's order")


def reference_indices(best: np.ndarray, vals: np.ndarray) -> np.ndarray:
    """The reference TopK order (largest first, ties to the smaller index)
    recomputed from the reference's per-anchor scores."""
    order = np.lexsort((np.arange(best.shape[1])[None, :].repeat(best.shape[0], 0), -best), axis=1)
    return order[:, : vals.shape[1]]
