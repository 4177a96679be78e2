#!/usr/bin/env python
"""Throughput benchmark of the SPINNV2 B200 CUDA target: ResNet-101 img/s at
batch 64 per GPU on 1/2/4/8 B200.

One step = one ResNet-101 v1.5 forward pass (fp32 activations, 3xTF32 conv
math by default) over a batch of 64 synthetic N(0,1) 3x224x224 images with
seeded random-init weights, executed by libspkv2_runtime.so.  Multi-GPU is
batch-sharded inference with no data-path collective: every rank holds its
own SPK, weights and arenas.  The headline runs 64 images per rank (weak
scaling); the `strong` sub-object splits one global batch of 64 (and 256)
into contiguous ceil(B/N) slices, one per rank.  torch.distributed only
provides the start/stop barrier and the max-over-ranks of the timed region.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line on rank 0.  On one GPU the line also carries the other
figures of the north star: plain TF32 mode, INT8 ResNet-50 at batch 256, the
YOLOv10n-style detector at batch 1 and 64, the memory-bound ops of that
detector, the bs1 latency and the reference CPU runtime at all host cores and
at one thread.  --impl reference times the reference SPINNV2 CPU runtime
(oracle/_ref, built from the reference's own sources) on the host cores for
the same config and batch.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def metric_name(args) -> str:
    """The fp32 headline metric, or the INT8 ResNet-50 line (--int8)."""
    if args.int8:
        return f"ResNet-50 INT8 img/s (bs{args.batch} per GPU)"
    return f"ResNet-101 img/s (bs{args.batch} per GPU)"


def peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


class ClockSampler:
    """SM clock and clock-event reasons sampled DURING the timed region: NVML
    polled every 10 ms from a thread (the device found by the UUID CUDA
    reports, so it is the GPU this rank runs on even under
    CUDA_VISIBLE_DEVICES), else `nvidia-smi -lms 200`.  Read-only."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, cuda_device: int, period_s: float = 0.01) -> None:
        self.dev = cuda_device
        self.period = period_s
        self.proc = None
        self.nvml = None
        self.lines: list[str] = []
        self.samples: list[tuple[float, float, int]] = []
        self.stop_evt = threading.Event()

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
        return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)

    def start(self) -> None:
        try:
            self.nvml, handle = self._nvml_handle()
            self.thread = threading.Thread(target=self._poll, args=(handle,), daemon=True)
            self.thread.start()
            return
        except Exception:  # noqa: BLE001 - no NVML binding or device: fall back to nvidia-smi
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.dev)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _poll(self, handle) -> None:
        nv = self.nvml
        while not self.stop_evt.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM)),
                                     float(nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM)),
                                     int(nv.nvmlDeviceGetCurrentClocksEventReasons(handle))))
            except Exception:  # noqa: BLE001
                break
            self.stop_evt.wait(self.period)

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.nvml is not None:
            self.stop_evt.set()
            self.thread.join(timeout=5)
            sm = [x[0] for x in self.samples]
            reasons = {name for _, _, bits in self.samples for name, bit in self.REASONS if bits & bit}
            return {"sm_mhz": statistics.median(sm) if sm else None,
                    "sm_max_mhz": max(x[1] for x in self.samples) if sm else None,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml 10 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi 200 ms"}


def conv_flops(pkg, int8_only: bool = False) -> tuple[float, list[int]]:
    """2 x MACs of the (int8) convs of one step, and their node ids."""
    total, ids = 0.0, []
    for n in pkg.nodes:
        if n.op_type == "Conv" and (not int8_only or pkg.tensors[n.inputs[1]].np_dtype == np.int8):
            w = pkg.tensors[n.inputs[1]].shape
            y = pkg.tensors[n.outputs[0]].shape
            total += 2.0 * y[0] * y[1] * y[2] * y[3] * w[1] * w[2] * w[3]
            ids.append(n.id)
    return total, ids


def node_bytes(pkg, ids, skip_weights: bool = False) -> int:
    """Algorithmic HBM bytes of the given nodes: every input (activation,
    weights, bias, residual) read once and every output written once."""
    total = 0
    for n in pkg.nodes:
        if n.id in ids:
            for t in list(n.inputs) + list(n.outputs):
                if t >= 0:
                    ten = pkg.tensors[t]
                    if skip_weights and ten.role_name == "weight":
                        continue
                    total += int(np.prod(ten.shape)) * np.dtype(ten.np_dtype).itemsize
    return total


# DRAM traffic of the conv kernels relative to their algorithmic bytes, from
# ncu captures of single launches on small cases (one kernel, one launch per
# capture, a process of a few hundred MB; cold cache, so the input is read
# from DRAM).  traffic_step = ratio x the step's algorithmic conv bytes.
# Keyed by conv math; each entry names its capture.
CONV_TRAFFIC_RATIO = {
    "3xtf32": (0.74, "the layer-3 3x3 (0.63) and 1x1 (0.85) convs of ResNet-101 bs64, each captured as a single "
                     "launch of the sweep configs conv3x3_256_14 / conv1x1_1024_256_14 at batch 64 "
                     "(profiles/conv_tc_layer3_bs64.md)"),
    "tf32": (None, "not captured"),
    "int8": (None, "not captured"),
}


def use_all_host_threads() -> None:
    """OpenMP threads for the reference CPU runtime: every host core (torchrun
    exports OMP_NUM_THREADS=1 to its workers), unless SPKV2_REF_THREADS says
    otherwise.  Set before the reference library is first loaded."""
    os.environ["OMP_NUM_THREADS"] = os.environ.get("SPKV2_REF_THREADS", str(os.cpu_count() or 1))


def reference_package(config: str, batch: int) -> bytes:
    """The config packaged for the reference CPU runtime.  The package
    checksum is computed by the compiler's pure-Python FNV-1a, so the
    reference arm never maps this repository's CUDA library."""
    from spinnv2_b200.compiler import pipeline, spk_writer

    spk_writer.NATIVE_FNV = False
    return pipeline.compile_config(config, batch, targets=("cpu_generic_x86",))["cpu_generic_x86"]


def cpu_oracle_int8_throughput(config: str, batch: int, seconds: float, max_steps: int | None = None) -> dict:
    """INT8 CPU baseline: the reference's INT8 conv kernel is ARM-dotprod only
    (on x86 it falls back to the fp32 loop over int8 bytes), so the INT8
    baseline is the oracle's C restatement of the INT8 contract (OpenMP over
    output channels) running the same package, timed on a bounded sample."""
    from oracle import harness
    from spinnv2_b200.compiler import pipeline, spk_writer
    from spinnv2_b200.spk import read_spk

    spk_writer.NATIVE_FNV = False
    spk = pipeline.compile_config(config, batch, targets=("cuda_b200",), int8=True)["cuda_b200"]
    pkg = read_spk(spk)
    x = np.random.default_rng(1).standard_normal(pkg.inputs[0].shape, dtype=np.float32)
    harness.run_spk(pkg, [x])
    times = []
    start = time.perf_counter()
    while time.perf_counter() - start < seconds and (max_steps is None or len(times) < max_steps):
        t0 = time.perf_counter()
        harness.run_spk(pkg, [x])
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    return {"value": batch / per, "step_s": per, "steps": len(times), "times": times}


def cpu_reference_throughput(config: str, batch: int, seconds: float, max_steps: int | None = None) -> dict:
    """Reference CPU runtime (oracle/_ref) img/s on a bounded sample."""
    from oracle import refrt
    from spinnv2_b200.spk import read_spk

    spk = reference_package(config, batch)
    pkg = read_spk(spk)
    x = np.random.default_rng(1).standard_normal(pkg.inputs[0].shape, dtype=np.float32)
    rt = refrt.RefRuntime(spk, [(tuple(t.shape), t.np_dtype) for t in pkg.outputs])
    rt.run(x)  # warm-up (lazy weight packing)
    times = []
    start = time.perf_counter()
    while time.perf_counter() - start < seconds and (max_steps is None or len(times) < max_steps):
        t0 = time.perf_counter()
        rt.run(x)
        times.append(time.perf_counter() - t0)
    rt.close()
    per = statistics.median(times)
    return {"value": batch / per, "step_s": per, "steps": len(times), "times": times}


def cpu_one_thread(config: str, seconds: float) -> dict | None:
    """The reference CPU runtime with one OpenMP thread (a child process, so
    the thread count is fixed before the runtime loads), batch 1."""
    code = ("import json, sys; sys.path.insert(0, %r); import bench; "
            "r = bench.cpu_reference_throughput(%r, 1, %r); r.pop('times'); print(json.dumps(r))"
            % (str(REPO), config, seconds))
    env = dict(os.environ, OMP_NUM_THREADS="1", SPKV2_REF_THREADS="1")
    try:
        out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                             timeout=seconds * 6 + 120, check=True)
        return json.loads(out.stdout.strip().splitlines()[-1])
    except (subprocess.SubprocessError, ValueError, IndexError):
        return None


def run_reference_arm(args, group) -> None:
    """The reference CPU runtime on the host cores, on the GPU arm's config
    and batch: every step runs the whole batch (rank 0 only)."""
    if group.rank != 0:
        return
    use_all_host_threads()
    if args.int8:
        res = cpu_oracle_int8_throughput(args.config, args.batch, seconds=1e9, max_steps=args.warmup + args.steps)
        times = res["times"]
    else:
        from oracle import refrt
        from spinnv2_b200.spk import read_spk

        spk = reference_package(args.config, args.batch)
        pkg = read_spk(spk)
        x = np.random.default_rng(1).standard_normal(pkg.inputs[0].shape, dtype=np.float32)
        rt = refrt.RefRuntime(spk, [(tuple(t.shape), t.np_dtype) for t in pkg.outputs])
        times = []
        for _ in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            rt.run(x)
            times.append(time.perf_counter() - t0)
        rt.close()
    timed = times[args.warmup:] or times
    ms = 1000.0 * sum(timed) / len(timed)
    value = args.batch / (ms / 1000.0)
    line = {
        "impl": "reference", "metric": metric_name(args), "value": value, "unit": "img/s", "n_gpus": args.gpus,
        "steps": len(timed), "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8" if args.int8 else "f32", "data": "synthetic",
        "config": {"workload": workload_name(args), "model": args.config, "global_batch": args.batch,
                   "runtime": ("INT8 oracle (C restatement of the INT8 contract, OpenMP); the reference INT8 kernel "
                               "is ARM-dotprod only") if args.int8 else
                   "reference cpu_generic (AVX2/FMA, OpenMP), BNNS token removed from the profile"},
        "cpu_baseline": {"value": value, "unit": "img/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
                         "kind": "port" if args.int8 else "reference",
                         "sample": f"the full batch of {args.batch} per step, {len(timed)} timed steps"},
        "e2e": {"value": value, "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_name(args) -> str:
    if args.int8:
        return f"{args.config} INT8 forward, batch {args.batch} per GPU, 224x224, int8 activations between convs"
    return f"{args.config} v1.5 forward, batch {args.batch} per GPU, 224x224, fp32 activations, conv math {args.math}"


# ---------------------------------------------------------------- GPU timing


def time_replays(rt, steps: int, warmup: int, flush, stream) -> list[float]:
    """Device ms of `steps` graph replays (after `warmup`), each bracketed by
    CUDA events on the runtime's own stream, with an L2 flush (a 256 MiB
    write) between steps."""
    import torch

    for _ in range(warmup):
        rt.run_async()
    rt.synchronize()
    torch.cuda.synchronize()
    evs = []
    with torch.cuda.stream(stream):
        for _ in range(steps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            rt.run_async()
            e.record(stream)
            evs.append((s, e))
    rt.synchronize()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def node_shares(rt, repeats: int = 3) -> np.ndarray:
    """Per-node device ms of eager, event-bracketed runs (mean of `repeats`)."""
    return np.stack([rt.profile_nodes() for _ in range(repeats)]).mean(axis=0)


def conv_roofline(rt, pkg, ms_per_step: float, int8: bool, math_label: str) -> dict:
    """Conv roofline of a graph-replayed step: the conv nodes' share of the
    eager per-node device time, times the replayed step time, gives their
    time in the step; achieved = conv FLOPs (or int8 ops) / that time."""
    flops, ids = conv_flops(pkg, int8_only=int8)
    node_ms = node_shares(rt)
    share = float(node_ms[ids].sum() / max(node_ms.sum(), 1e-9))
    conv_ms = share * ms_per_step
    pk, basis = peaks()
    if int8:
        peak, unit = pk["bf16_tflops"] * 2.0, "TOPS"
        peak_basis = f"INT8 dense = bf16 {basis} {pk['bf16_tflops']} x 2 (derived)"
    else:
        peak, unit = pk["bf16_tflops"] / 2.0, "TFLOP/s"
        peak_basis = f"TF32 dense = bf16 {basis} {pk['bf16_tflops']} / 2 (derived)"
    achieved = flops / (conv_ms / 1000.0) / 1e12
    alg = node_bytes(pkg, ids)
    key = "int8" if int8 else math_label
    ratio, capture = CONV_TRAFFIC_RATIO.get(key, (None, "not captured"))
    out = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
           "traffic": alg * ratio if ratio else None,
           "traffic_basis": (f"scaled: {ratio:.3f} x the step's algorithmic conv bytes, the DRAM/algorithmic "
                             f"ratio of {capture}") if ratio else capture,
           "algorithmic_bytes_per_step": alg,
           "kernel": ("all int8 Conv launches" if int8 else "all Conv launches") + " of one graph-replayed step",
           "flops_per_step": flops, "conv_share_of_step": share, "conv_ms_per_step": conv_ms,
           "peak_basis": peak_basis, "conv_variants": sorted({rt.node_variant(i) for i in ids})}
    if math_label == "3xtf32" and not int8:
        # Each product is three TF32 MMAs: the tensor pipe's TF32 work rate.
        out["tensor_pipe_frac"] = 3.0 * achieved / peak
    return out


def device_run(config: str, batch: int, args, local: int, math_mode: int | None, int8: bool = False,
               want_roofline: bool = False, math_label: str = "3xtf32", flush=None) -> dict:
    """Graph-replayed throughput of one config with the input resident in HBM."""
    import torch

    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import Runtime

    spk = pipeline.compile_config(config, batch, targets=("cuda_b200",), seed=0, int8=int8)["cuda_b200"]
    with Runtime(spk, device=local, math_mode=math_mode, graph=True) as rt:
        pkg = rt.package
        x = np.random.default_rng(5).standard_normal(pkg.inputs[0].shape, dtype=np.float32)
        if config == "yolo_style":
            x = np.random.default_rng(5).random(pkg.inputs[0].shape, dtype=np.float32)
        d_in = torch.from_numpy(x).cuda(local)
        rt.bind_input(0, d_in.data_ptr())
        stream = torch.cuda.ExternalStream(rt.stream())
        step_ms = time_replays(rt, args.steps, args.warmup, flush, stream)
        ms = sum(step_ms) / len(step_ms)
        out = {"value": batch / (ms / 1000.0), "unit": "img/s", "ms_per_step": ms, "batch": batch,
               "steps": args.steps, "gpu_launches_per_step": rt.launches_per_run()}
        if want_roofline:
            out["roofline"] = conv_roofline(rt, pkg, ms, int8, math_label)
    return out


def latency_bs1(args, local: int, math_mode: int) -> dict:
    """bs1 latency through the public API, the reference's `spkv2_bench`
    protocol: warm-up runs, then `runs` timed spkv2_run calls, each copying the
    input from pinned host memory, replaying the captured graph and copying
    the output back (spkv2_run synchronises); p50/p90 of the per-run wall
    time."""
    import torch

    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import Runtime

    spk1 = pipeline.compile_config(args.config, 1, targets=("cuda_b200",), seed=0, int8=args.int8)["cuda_b200"]
    rt = Runtime(spk1, device=local, math_mode=math_mode, graph=True)
    in_t, out_t = rt.package.inputs[0], rt.package.outputs[0]
    x1 = np.random.default_rng(2).standard_normal(in_t.shape, dtype=np.float32)
    h_in = torch.from_numpy(x1).pin_memory()
    h_out = torch.empty(tuple(out_t.shape), dtype=torch.float32).pin_memory()
    rt.bind_input(0, h_in.data_ptr())
    rt.bind_output(0, h_out.data_ptr())
    for _ in range(20):
        rt._check(rt.lib.spkv2_run(rt.ctx), "run")
    times = []
    for _ in range(args.latency_runs):
        t0 = time.perf_counter()
        rt._check(rt.lib.spkv2_run(rt.ctx), "run")
        times.append(time.perf_counter() - t0)
    rt.close()
    times.sort()
    return {"p50_ms": 1000.0 * statistics.median(times), "p90_ms": 1000.0 * times[int(0.9 * (len(times) - 1))],
            "min_ms": 1000.0 * times[0], "runs": len(times), "batch": 1,
            "path": "spkv2_run: pinned host input -> graph replay -> pinned host output"}


def memory_bound(batch: int, local: int) -> dict:
    """Memory-bound ops (every node that is not a Conv/Gemm) of the
    YOLOv10n-style config: per node, algorithmic bytes (every input and
    output tensor read/written once) / device time (per-node CUDA events,
    mean of 5 passes), aggregated per op type, against the measured HBM copy
    bandwidth."""
    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import Runtime

    spk = pipeline.compile_config("yolo_style", batch, targets=("cuda_b200",), seed=0)["cuda_b200"]
    with Runtime(spk, device=local, graph=False) as rt:
        pkg = rt.package
        x = np.random.default_rng(3).random(pkg.inputs[0].shape, dtype=np.float32)
        rt.set_input(0, x)
        rt.run()
        ms = node_shares(rt, 5)
        per_op: dict[str, list[float]] = {}
        nodes = []
        for n in pkg.nodes:
            if n.op_type in ("Conv", "Gemm") or ms[n.id] <= 0:
                continue
            nbytes = node_bytes(pkg, [n.id], skip_weights=True)
            acc = per_op.setdefault(n.op_type, [0, 0.0, 0.0])
            acc[0] += 1
            acc[1] += nbytes
            acc[2] += float(ms[n.id])
            nodes.append((nbytes / (ms[n.id] * 1e-3) / 1e9, n.op_type, n.id, nbytes, float(ms[n.id]),
                          rt.node_variant(n.id)))
    pk, basis = peaks()
    tot_b = sum(v[1] for v in per_op.values())
    tot_ms = sum(v[2] for v in per_op.values())
    big = [r for r in nodes if r[3] >= 64 * 2**20]  # tensors well above L2
    gbs = tot_b / (tot_ms * 1e-3) / 1e9
    return {
        "metric": "memory-bound op GB/s (YOLOv10n-style, non-conv nodes)", "unit": "GB/s", "value": gbs,
        "workload": f"yolo_style 640x640 fp32 forward, batch {batch}", "nodes": len(nodes),
        "peak": pk["hbm_gbs"], "peak_basis": f"HBM copy, {basis}", "frac": gbs / pk["hbm_gbs"],
        "ms_per_step": tot_ms,
        "per_op": {k: {"nodes": v[0], "bytes": int(v[1]), "ms": v[2], "gbs": v[1] / (v[2] * 1e-3) / 1e9}
                   for k, v in sorted(per_op.items(), key=lambda kv: -kv[1][2])},
        "nodes_over_64MiB_gbs": (sum(r[3] for r in big) / (sum(r[4] for r in big) * 1e-3) / 1e9) if big else None,
        "top_nodes": [{"op": r[1], "node": r[2], "bytes": r[3], "ms": r[4], "gbs": r[0], "variant": r[5]}
                      for r in sorted(nodes, key=lambda r: -r[4])[:8]],
    }


def node_times(config: str, batch: int, local: int, int8: bool, math_mode: int | None) -> dict:
    """Per-node device time of one config (eager, per-node CUDA events, mean
    of 5 passes): the conv nodes with their shapes, FLOP rate and kernel
    variant, and every other node's time.  A diagnostic line, not a bench
    figure: no graph replay, no PDL overlap between nodes."""
    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import Runtime

    spk = pipeline.compile_config(config, batch, targets=("cuda_b200",), int8=int8)["cuda_b200"]
    kw = {} if math_mode is None else {"math_mode": math_mode}
    with Runtime(spk, device=local, graph=False, **kw) as rt:
        pkg = rt.package
        x = np.random.default_rng(1).standard_normal(pkg.inputs[0].shape, dtype=np.float32)
        rt.set_input(0, x)
        rt.run()
        ms = node_shares(rt, 5)
        rows = []
        for n in pkg.nodes:
            row = {"node": n.id, "op": n.op_type, "ms": float(ms[n.id]), "variant": rt.node_variant(n.id)}
            if n.op_type == "Conv":
                w = pkg.tensors[n.inputs[1]].shape
                y = pkg.tensors[n.outputs[0]].shape
                flop = 2.0 * y[0] * y[1] * y[2] * y[3] * w[1] * w[2] * w[3]
                row.update({"shape": f"{w[1]}->{w[0]} k{w[2]}x{w[3]} out{y[2]}x{y[3]}",
                            "tflops": flop / (float(ms[n.id]) * 1e-3) / 1e12 if ms[n.id] > 0 else None})
            rows.append(row)
    return {"config": config, "batch": batch, "int8": int8, "total_ms": float(sum(r["ms"] for r in rows)),
            "nodes": rows}


def strong_scaling(args, group, math_mode: int, flush) -> dict:
    """One global batch split into contiguous ceil(B/N) slices, one per rank
    (the per-rank form of ShardedRuntime): each rank compiles and prepares
    its slice, then every step replays it; device time per step is the max
    over ranks.  Two figures per global batch: inputs resident in HBM, and
    end to end through spkv2_run with the rank's slice copied from pinned
    host memory and the outputs copied back."""
    import torch

    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import Runtime

    out = {}
    for gb in args.strong_batches:
        start, count = group.slice(gb)
        spk = pipeline.compile_config(args.config, max(count, 1), targets=("cuda_b200",), seed=0)["cuda_b200"]
        with Runtime(spk, device=group.local_rank, math_mode=math_mode, graph=True) as rt:
            pkg = rt.package
            x = np.random.default_rng(40 + group.rank).standard_normal(pkg.inputs[0].shape, dtype=np.float32)
            d_in = torch.from_numpy(x).cuda(group.local_rank)
            rt.bind_input(0, d_in.data_ptr())
            stream = torch.cuda.ExternalStream(rt.stream())
            group.barrier()
            step_ms = time_replays(rt, args.steps, args.warmup, flush, stream) if count else [0.0] * args.steps
            dev_ms = group.max(sum(step_ms)) / args.steps
            h_in = torch.from_numpy(x).pin_memory()
            h_out = [torch.empty(tuple(t.shape), dtype=torch.float32).pin_memory() for t in pkg.outputs]
            rt.bind_input(0, h_in.data_ptr())
            for k, o in enumerate(h_out):
                rt.bind_output(k, o.data_ptr())
            for _ in range(2):
                rt._check(rt.lib.spkv2_run(rt.ctx), "run")
            group.barrier()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                if count:
                    rt._check(rt.lib.spkv2_run(rt.ctx), "run")
            e2e_s = group.max(time.perf_counter() - t0)
        out[f"global_batch_{gb}"] = {
            "value": gb * args.steps / (dev_ms * args.steps / 1000.0), "unit": "img/s", "ms_per_step": dev_ms,
            "e2e_value": gb * args.steps / e2e_s, "per_gpu_batch": count, "n_gpus": group.world,
            "slices": "contiguous ceil(B/N) per rank, one SPK per slice size"}
    return out


def run_gpu_arm(args, group) -> None:
    import torch

    world, rank, local = group.world, group.rank, group.local_rank

    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import MATH_3XTF32, MATH_FP32, MATH_SPEC, MATH_TF32, Runtime

    math_mode = {"spec": MATH_SPEC, "3xtf32": MATH_3XTF32, "tf32": MATH_TF32, "fp32": MATH_FP32}[args.math]
    math_label = "3xtf32" if args.math in ("spec", "3xtf32") else args.math
    torch.cuda.set_device(local)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local}")  # > 126 MB L2
    spk = pipeline.compile_config(args.config, args.batch, targets=("cuda_b200",), seed=0, int8=args.int8)["cuda_b200"]
    rt = Runtime(spk, device=local, math_mode=math_mode, graph=True)
    pkg = rt.package
    in_t, out_t = pkg.inputs[0], pkg.outputs[0]
    rng = np.random.default_rng(1 + rank)
    x = rng.standard_normal(in_t.shape, dtype=np.float32)
    stream = torch.cuda.ExternalStream(rt.stream())

    # ---- device-resident timing (inputs already in HBM) ----
    d_in = torch.from_numpy(x).cuda(local)
    rt.bind_input(0, d_in.data_ptr())
    for _ in range(args.warmup):
        rt.run_async()
    rt.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    group.barrier()
    step_ms = time_replays(rt, args.steps, 0, flush, stream)
    group.barrier()
    clocks = sampler.stop()
    total_ms = group.max(sum(step_ms))
    ms_per_step = total_ms / args.steps
    value = world * args.batch * args.steps / (total_ms / 1000.0)
    roof = conv_roofline(rt, pkg, ms_per_step, args.int8, math_label)
    launches = rt.launches_per_run() * args.steps

    # ---- end to end through the public API: pinned host in/out, spkv2_run ----
    h_in = torch.from_numpy(x).pin_memory()
    h_out = torch.empty(tuple(out_t.shape), dtype=torch.float32).pin_memory()
    rt.bind_input(0, h_in.data_ptr())
    rt.bind_output(0, h_out.data_ptr())
    for _ in range(max(args.warmup, 2)):
        rt._check(rt.lib.spkv2_run(rt.ctx), "run")
    group.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        rt._check(rt.lib.spkv2_run(rt.ctx), "run")
    e2e_s = group.max(time.perf_counter() - t0)
    e2e_value = world * args.batch * args.steps / e2e_s
    rt.close()
    del d_in
    lat = latency_bs1(args, local, math_mode)  # every rank, so the ranks stay in step
    strong = strong_scaling(args, group, math_mode, flush) if not args.int8 and args.strong_batches else None

    extras = {}
    if world == 1 and not args.int8 and not args.no_extras:
        extras["tf32_mode"] = device_run(args.config, args.batch, args, local, MATH_TF32, want_roofline=True,
                                         math_label="tf32", flush=flush)
        extras["int8"] = device_run("resnet50", args.int8_batch, args, local, None, int8=True, want_roofline=True,
                                    flush=flush)
        extras["int8"]["workload"] = f"resnet50 INT8 forward, batch {args.int8_batch}"
        extras["yolo"] = {f"bs{b}": device_run("yolo_style", b, args, local, math_mode, flush=flush)
                          for b in (1, args.mb_batch)}
        extras["memory_bound"] = memory_bound(args.mb_batch, local)

    if rank == 0:
        line = {
            "metric": metric_name(args), "value": value, "unit": "img/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8" if args.int8 else "f32", "data": "synthetic",
            "config": {"workload": workload_name(args), "model": args.config, "global_batch": args.batch * world,
                       "per_gpu_batch": args.batch, "seq_len": None,
                       "parallelism": f"batch-sharded x{world}, no collectives",
                       "l2": "flushed between steps (256 MiB write)"},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": "img/s", "h2d_bytes_per_step": int(x.nbytes),
                    "d2h_bytes_per_step": int(np.prod(out_t.shape) * 4)},
            "gpu_launches": int(launches),
            "latency_bs1": lat,
            "roofline": roof,
        }
        if strong:
            line["strong"] = strong
        line.update(extras)
        if world == 1 and not args.no_cpu_baseline:
            use_all_host_threads()
            timer = cpu_oracle_int8_throughput if args.int8 else cpu_reference_throughput
            cb = timer(args.config, 1, seconds=args.cpu_seconds)
            line["cpu_baseline"] = {"value": cb["value"], "unit": "img/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
                                    "kind": "port" if args.int8 else "reference",
                                    "sample": f"batch 1, {cb['steps']} runs over ~{args.cpu_seconds:.0f} s",
                                    "p50_ms_bs1": 1000.0 * cb["step_s"]}
            if not args.int8:
                one = cpu_one_thread(args.config, args.cpu_seconds)
                if one:
                    line["cpu_baseline"]["one_thread"] = {
                        "value": one["value"], "unit": "img/s", "cores": 1, "p50_ms_bs1": 1000.0 * one["step_s"],
                        "sample": f"batch 1, {one['steps']} runs over ~{args.cpu_seconds:.0f} s"}
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="resnet101")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--math", default="spec", choices=["spec", "3xtf32", "tf32", "fp32"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="headline only (no TF32/INT8/YOLO/memory-bound)")
    ap.add_argument("--latency-runs", type=int, default=200, help="timed spkv2_run calls for the bs1 latency")
    ap.add_argument("--strong-batches", type=int, nargs="*", default=[64, 256],
                    help="global batches split across the ranks (strong scaling)")
    ap.add_argument("--memory-bound", action="store_true", help="only the YOLOv10n-style memory-bound line")
    ap.add_argument("--mb-batch", type=int, default=64)
    ap.add_argument("--int8-batch", type=int, default=256)
    ap.add_argument("--int8", action="store_true", help="INT8 quantised network (use with --config resnet50)")
    ap.add_argument("--nodes", action="store_true",
                    help="only per-node device times of --config at --batch (eager, per-node events; diagnostic)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    from spinnv2_b200.shard import RankGroup

    if args.impl == "reference":
        # Host cores only, rank 0 alone: no process group is needed.
        env = os.environ
        group = RankGroup(int(env.get("WORLD_SIZE", "1")), int(env.get("RANK", "0")), int(env.get("LOCAL_RANK", "0")),
                          None)
    else:
        group = RankGroup.from_env(backend="nccl", timeout_s=300)
    try:
        if args.impl == "reference":
            run_reference_arm(args, group)
        elif args.memory_bound:
            if group.rank == 0:
                print(json.dumps(memory_bound(args.mb_batch, group.local_rank)), flush=True)
        elif args.nodes:
            if group.rank == 0:
                from spinnv2_b200.runtime import MATH_3XTF32, MATH_FP32, MATH_TF32

                mm = {"spec": None, "3xtf32": MATH_3XTF32, "tf32": MATH_TF32, "fp32": MATH_FP32}[args.math]
                print(json.dumps(node_times(args.config, args.batch, group.local_rank, args.int8, mm)), flush=True)
        else:
            run_gpu_arm(args, group)
    finally:
        group.close()


if __name__ == "__main__":
    main()
