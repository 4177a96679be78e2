#!/usr/bin/env python
"""Throughput benchmark of the SPINNV2 B200 CUDA target: ResNet-101 img/s at
batch 64 per GPU on 1/2/4/8 B200.

One step = one ResNet-101 v1.5 forward pass (fp32 activations, 3xTF32 conv
math by default) over a batch of 64 synthetic N(0,1) 3x224x224 images with
seeded random-init weights, executed by libspkv2_runtime.so.  Multi-GPU is
batch-sharded inference with no data-path collective: every rank holds its
own SPK, weights and arenas and runs its own batch of 64 (weak scaling);
torch.distributed only provides the start/stop barrier and the max-over-ranks
of the timed region.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line on rank 0.  --impl reference times the reference
SPINNV2 CPU runtime (oracle/_ref, built from the reference's own sources) on
the host cores for the same config, on a bounded batch sample per step.
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

METRIC = "ResNet-101 img/s (bs64 per GPU)"


def metric_name(args) -> str:
    """The fp32 headline metric, or the INT8 ResNet-50 line (--int8)."""
    if args.int8:
        return f"ResNet-50 INT8 img/s (bs{args.batch} per GPU)"
    return METRIC
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


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


def conv_bytes(pkg, ids: list[int]) -> int:
    """Algorithmic HBM bytes of the given conv nodes: every input (activation,
    weights, bias, residual) read once and the output written once."""
    total = 0
    for n in pkg.nodes:
        if n.id in ids:
            for t in list(n.inputs) + list(n.outputs):
                if t >= 0:
                    ten = pkg.tensors[t]
                    total += int(np.prod(ten.shape)) * np.dtype(ten.np_dtype).itemsize
    return total


# DRAM bytes (read + write) of the conv launches of one step, each from one
# ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of the second
# pass through the network:
#   fp32: ncu ... -c 560 python bench.py --steps 2 --warmup 3 --no-cpu-baseline --latency-runs 5
#         (the 105 conv launches of launches 433..541)
#   int8: ncu ... -k regex:conv_i8 -s 52 -c 52 python bench.py --config resnet50 --int8 --batch 256
#         --steps 2 --warmup 3 --no-cpu-baseline --latency-runs 5
# Keyed by the workload it was measured on; other workloads report null.
MEASURED_CONV_TRAFFIC = {
    ("resnet101", 64, "3xtf32", False): 6591.0e6 + 1543.6e6,
    # the 52 int8 conv launches of one ResNet-50 bs256 step
    ("resnet50", 256, "int8", True): 3861.2e6 + 1179.7e6,
}


def use_all_host_threads() -> None:
    """OpenMP threads for the reference CPU runtime: every host core (torchrun
    exports OMP_NUM_THREADS=1 to its workers), unless SPKV2_REF_THREADS says
    otherwise.  Set before the reference library is first loaded."""
    os.environ["OMP_NUM_THREADS"] = os.environ.get("SPKV2_REF_THREADS", str(os.cpu_count() or 1))


def cpu_oracle_int8_throughput(config: str, batch: int, seconds: float, max_steps: int | None = None) -> dict:
    """INT8 CPU baseline: the reference's INT8 conv kernel is ARM-dotprod only
    (on x86 it falls back to the fp32 loop over int8 bytes), so the INT8
    baseline is the oracle's C restatement of the INT8 contract (OpenMP over
    output channels) running the same package, timed on a bounded sample."""
    from oracle import harness
    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.spk import read_spk

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
    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.spk import read_spk

    spk = pipeline.compile_config(config, batch, targets=("cpu_generic_x86",))["cpu_generic_x86"]
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


def run_reference_arm(args, group) -> None:
    if group.rank != 0:
        return
    sample = min(args.batch, args.reference_sample)
    use_all_host_threads()
    timer = cpu_oracle_int8_throughput if args.int8 else cpu_reference_throughput
    res = timer(args.config, sample, seconds=1e9, max_steps=args.warmup + args.steps)
    timed = res["times"][args.warmup:] or res["times"]
    ms = 1000.0 * sum(timed) / len(timed)
    value = sample / (ms / 1000.0)
    line = {
        "impl": "reference", "metric": metric_name(args), "value": value, "unit": "img/s", "n_gpus": args.gpus,
        "steps": len(timed), "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8" if args.int8 else "f32", "data": "synthetic",
        "config": {"workload": f"{args.config} {'int8' if args.int8 else 'fp32'} forward, batch {args.batch}",
                   "model": args.config, "global_batch": args.batch, "sample_batch_per_step": sample,
                   "runtime": ("INT8 oracle (C restatement of the INT8 contract, OpenMP); the reference INT8 kernel "
                               "is ARM-dotprod only") if args.int8 else
                   "reference cpu_generic (AVX2/FMA, OpenMP), BNNS token removed from the profile"},
        "cpu_baseline": {"value": value, "unit": "img/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
                         "kind": "port" if args.int8 else "reference",
                         "sample": f"{sample} images per step, {len(timed)} steps"},
        "e2e": {"value": value, "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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


def run_memory_bound(args, group) -> None:
    """Memory-bound ops (every node that is not a Conv/Gemm) of the
    YOLOv10n-style config at `--mb-batch`: per node, algorithmic bytes (every
    input and output tensor read/written once) / device time (per-node CUDA
    events, mean of 5 passes), aggregated per op type, against the measured
    HBM copy bandwidth.  Rank 0 prints one JSON line."""
    if group.rank != 0:
        return
    import torch

    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import Runtime

    torch.cuda.set_device(group.local_rank)
    spk = pipeline.compile_config("yolo_style", args.mb_batch, targets=("cuda_b200",), seed=0)["cuda_b200"]
    with Runtime(spk, device=group.local_rank, graph=False) as rt:
        pkg = rt.package
        x = np.random.default_rng(3).random(pkg.inputs[0].shape, dtype=np.float32)
        rt.set_input(0, x)
        rt.run()
        ms = np.mean([rt.profile_nodes() for _ in range(5)], axis=0)
        per_op: dict[str, list[float]] = {}
        nodes = []
        for n in pkg.nodes:
            if n.op_type in ("Conv", "Gemm"):
                continue
            nbytes = 0
            for t in list(n.inputs) + list(n.outputs):
                if t >= 0 and pkg.tensors[t].role_name != "weight":
                    ten = pkg.tensors[t]
                    nbytes += int(np.prod(ten.shape)) * np.dtype(ten.np_dtype).itemsize
            if ms[n.id] <= 0:
                continue
            acc = per_op.setdefault(n.op_type, [0, 0.0, 0.0])
            acc[0] += 1
            acc[1] += nbytes
            acc[2] += float(ms[n.id])
            nodes.append((nbytes / (ms[n.id] * 1e-3) / 1e9, n.op_type, n.id, nbytes, float(ms[n.id]), rt.node_variant(n.id)))
    pk, basis = peaks()
    tot_b = sum(v[1] for v in per_op.values())
    tot_ms = sum(v[2] for v in per_op.values())
    big = [r for r in nodes if r[3] >= 64 * 2**20]  # tensors well above L2
    line = {
        "metric": "memory-bound op GB/s (YOLOv10n-style, non-conv nodes)", "unit": "GB/s",
        "value": tot_b / (tot_ms * 1e-3) / 1e9, "higher_is_better": True, "n_gpus": 1, "data": "synthetic",
        "config": {"workload": f"yolo_style 640x640 fp32 forward, batch {args.mb_batch}", "nodes": len(nodes)},
        "peak": {"value": pk["hbm_gbs"], "unit": "GB/s", "basis": f"HBM copy, {basis}"},
        "frac": tot_b / (tot_ms * 1e-3) / 1e9 / pk["hbm_gbs"],
        "per_op": {k: {"nodes": v[0], "bytes": int(v[1]), "ms": v[2], "gbs": v[1] / (v[2] * 1e-3) / 1e9}
                   for k, v in sorted(per_op.items(), key=lambda kv: -kv[1][2])},
        "nodes_over_64MiB_gbs": (sum(r[3] for r in big) / (sum(r[4] for r in big) * 1e-3) / 1e9) if big else None,
        "top_nodes": [{"op": r[1], "node": r[2], "bytes": r[3], "ms": r[4], "gbs": r[0], "variant": r[5]}
                      for r in sorted(nodes, key=lambda r: -r[4])[:12]],
    }
    print(json.dumps(line), flush=True)


def run_gpu_arm(args, group) -> None:
    import torch

    world, rank, local = group.world, group.rank, group.local_rank

    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import MATH_3XTF32, MATH_FP32, MATH_SPEC, MATH_TF32, Runtime

    math_mode = {"spec": MATH_SPEC, "3xtf32": MATH_3XTF32, "tf32": MATH_TF32, "fp32": MATH_FP32}[args.math]
    math_label = "3xtf32" if args.math in ("spec", "3xtf32") else args.math
    torch.cuda.set_device(local)
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
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local}")  # > 126 MB L2
    for _ in range(args.warmup):
        rt.run_async()
    rt.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    group.barrier()
    torch.cuda.synchronize()
    evs = []
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            rt.run_async()
            e.record(stream)
            evs.append((s, e))
    rt.synchronize()
    torch.cuda.synchronize()
    group.barrier()
    clocks = sampler.stop()
    step_ms = [s.elapsed_time(e) for s, e in evs]
    local_total_ms = sum(step_ms)
    total_ms = group.max(local_total_ms)
    ms_per_step = total_ms / args.steps
    value = world * args.batch * args.steps / (total_ms / 1000.0)

    # ---- roofline of the conv kernels (per-node events) ----
    flops, conv_ids = conv_flops(pkg, int8_only=args.int8)
    prof = np.stack([rt.profile_nodes() for _ in range(3)])
    node_ms = prof.mean(axis=0)
    conv_ms = float(node_ms[conv_ids].sum())
    pk, basis = peaks()
    if args.int8:
        peak, peak_unit = pk["bf16_tflops"] * 2.0, "TOPS"
        peak_basis = f"INT8 dense = bf16 {basis} {pk['bf16_tflops']} x 2 (derived)"
    else:
        peak, peak_unit = pk["bf16_tflops"] / 2.0, "TFLOP/s"
        peak_basis = f"TF32 dense = bf16 {basis} {pk['bf16_tflops']} / 2 (derived)"
    achieved = flops / (conv_ms / 1000.0) / 1e12
    variants = sorted({rt.node_variant(i) for i in conv_ids})
    alg_bytes = conv_bytes(pkg, conv_ids)
    eff_math = "int8" if args.int8 else math_label
    traffic = MEASURED_CONV_TRAFFIC.get((args.config, args.batch, eff_math, args.int8))

    # ---- end to end through the public API: pinned host in/out, spkv2_run ----
    rt2 = Runtime(spk, device=local, math_mode=math_mode, graph=True)
    h_in = torch.from_numpy(x).pin_memory()
    h_out = torch.empty(tuple(out_t.shape), dtype=torch.float32).pin_memory()
    rt2.bind_input(0, h_in.data_ptr())
    rt2.bind_output(0, h_out.data_ptr())
    for _ in range(max(args.warmup, 2)):
        rt2._check(rt2.lib.spkv2_run(rt2.ctx), "run")
    group.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        rt2._check(rt2.lib.spkv2_run(rt2.ctx), "run")
    e2e_s = group.max(time.perf_counter() - t0)
    e2e_value = world * args.batch * args.steps / e2e_s
    launches = rt.launches_per_run() * args.steps
    rt2.close()
    lat = latency_bs1(args, local, math_mode)  # every rank, so the ranks stay in step

    if rank == 0:
        line = {
            "metric": metric_name(args), "value": value, "unit": "img/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8" if args.int8 else "f32", "data": "synthetic",
            "config": {"workload": f"{args.config} v1.5 forward, batch {args.batch} per GPU, 224x224, " + (
                           "int8 activations between convs (fp32 first conv and head)" if args.int8 else
                           f"fp32 activations, conv math {args.math}"),
                       "model": args.config, "global_batch": args.batch * world, "per_gpu_batch": args.batch,
                       "seq_len": None, "parallelism": f"batch-sharded x{world}, no collectives",
                       "l2": "flushed between steps (256 MiB write)", "conv_variants": variants},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": "img/s", "h2d_bytes_per_step": int(x.nbytes),
                    "d2h_bytes_per_step": int(np.prod(out_t.shape) * 4)},
            "gpu_launches": int(launches),
            "latency_bs1": lat,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": peak_unit,
                         "frac": achieved / peak, "traffic": traffic,
                         "algorithmic_bytes_per_step": alg_bytes,
                         "kernel": ("all int8 Conv launches" if args.int8 else "all Conv launches") + " of one step",
                         "flops_per_step": flops, "conv_ms_per_step": conv_ms, "peak_basis": peak_basis},
        }
        if world == 1 and not args.no_cpu_baseline:
            use_all_host_threads()
            timer = cpu_oracle_int8_throughput if args.int8 else cpu_reference_throughput
            cb = timer(args.config, 1, seconds=args.cpu_seconds)
            line["cpu_baseline"] = {"value": cb["value"], "unit": "img/s", "cores": int(os.environ["OMP_NUM_THREADS"]),
                                    "kind": "port" if args.int8 else "reference",
                                    "sample": f"batch 1, {cb['steps']} runs over ~{args.cpu_seconds:.0f} s",
                                    "p50_ms_bs1": 1000.0 * cb["step_s"]}
        print(json.dumps(line), flush=True)
    rt.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)  # ~0.5 s timed at bs64 3xTF32
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="resnet101")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--math", default="spec", choices=["spec", "3xtf32", "tf32", "fp32"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--reference-sample", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--latency-runs", type=int, default=200, help="timed spkv2_run calls for the bs1 latency")
    ap.add_argument("--memory-bound", action="store_true", help="GB/s of the YOLOv10n-style non-conv ops instead")
    ap.add_argument("--mb-batch", type=int, default=64)
    ap.add_argument("--int8", action="store_true", help="INT8 quantised network (use with --config resnet50)")
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
            run_memory_bound(args, group)
        else:
            run_gpu_arm(args, group)
    finally:
        group.close()


if __name__ == "__main__":
    main()
