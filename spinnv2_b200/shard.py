"""Batch-sharded multi-GPU execution of SPK models.

The reference runtime is single-device: one context, one host thread
(`runtime/src/executor.c`, `spkv2_run`).  Inference over a batch shards with
no exchange step, so the multi-GPU target is N independent replicas, each
with its own SPK (SPK shapes are fixed, so one package per distinct slice
batch), weights, arenas and stream, and no collective on the data path:

* `batch_slices(batch, world)` - contiguous slices of ceil(batch / world).
* `ShardedRuntime` - one process driving several GPUs: one `Runtime` and one
  host thread per device.  Each thread binds its slice of the caller's host
  input and output arrays (staged host<->device copies inside `spkv2_run`,
  which releases the GIL), so outputs land at offset slice_start x
  per-image bytes with no gather.
* `RankGroup` - the one-process-per-GPU form (torchrun): rank r runs slice r;
  torch.distributed provides only the start/stop barrier and the
  max-over-ranks of timings (NCCL on GPUs, gloo on CPU).
"""

from __future__ import annotations

import datetime
import os
from concurrent.futures import ThreadPoolExecutor
from typing import Callable, Sequence

import numpy as np


def batch_slices(batch: int, world: int) -> list[tuple[int, int]]:
    """(start, count) per rank: contiguous slices of ceil(batch / world).

    Ranks past the end of the batch get count 0 (they hold no replica)."""
    if batch < 0 or world < 1:
        raise ValueError(f"batch {batch} / world {world}")
    per = -(-batch // world) if batch else 0
    out = []
    for r in range(world):
        start = min(r * per, batch)
        out.append((start, max(0, min(per, batch - start))))
    return out


class ShardedRuntime:
    """Batch-sharded inference over several GPUs from one process.

    `spk_for_batch(n)` returns the SPK package for a slice of n images (for
    example `lambda n: pipeline.compile_config("resnet101", n)["cuda_b200"]`);
    it is called once per distinct slice size.  `runtime_factory` builds the
    per-device runtime (default `spinnv2_b200.runtime.Runtime`)."""

    def __init__(self, spk_for_batch: Callable[[int], bytes], batch: int, devices: Sequence[int], *,
                 math_mode: int | None = None, graph: bool = True, runtime_factory=None) -> None:
        if not devices:
            raise ValueError("no devices")
        if runtime_factory is None:
            from .runtime import Runtime as runtime_factory
        self.batch = batch
        self.devices = list(devices)
        self.slices = [s for s in batch_slices(batch, len(self.devices))]
        packages: dict[int, bytes] = {}
        self.runtimes = []
        for (start, count), dev in zip(self.slices, self.devices):
            if count == 0:
                self.runtimes.append(None)
                continue
            if count not in packages:
                packages[count] = spk_for_batch(count)
            self.runtimes.append(runtime_factory(packages[count], device=dev, math_mode=math_mode, graph=graph))
        first = next(rt for rt in self.runtimes if rt is not None)
        self.inputs = first.package.inputs
        self.outputs = first.package.outputs
        self._pool = ThreadPoolExecutor(max_workers=len(self.devices), thread_name_prefix="spkv2-shard")

    @staticmethod
    def _per_image(shape: Sequence[int]) -> int:
        return int(np.prod(shape[1:])) if len(shape) > 1 else 1

    def run(self, *inputs: np.ndarray) -> list[np.ndarray]:
        """Full-batch inputs (batch-major) -> full-batch outputs."""
        if len(inputs) != len(self.inputs):
            raise ValueError(f"expected {len(self.inputs)} inputs")
        full_in = []
        for t, x in zip(self.inputs, inputs):
            a = np.ascontiguousarray(x, dtype=t.np_dtype)
            if a.shape[0] != self.batch or a.shape[1:] != tuple(t.shape[1:]):
                raise ValueError(f"input {t.name}: expected batch {self.batch} x {tuple(t.shape[1:])}, got {a.shape}")
            full_in.append(a)
        full_out = [np.empty((self.batch, *t.shape[1:]), dtype=t.np_dtype) for t in self.outputs]

        def work(i: int) -> None:
            rt = self.runtimes[i]
            start, count = self.slices[i]
            if rt is None:
                return
            for k, a in enumerate(full_in):
                rt.bind_input(k, a.ctypes.data + start * self._per_image(a.shape) * a.itemsize)
            for k, o in enumerate(full_out):
                rt.bind_output(k, o.ctypes.data + start * self._per_image(o.shape) * o.itemsize)
            rt._check(rt.lib.spkv2_run(rt.ctx), "run")

        futures = [self._pool.submit(work, i) for i in range(len(self.runtimes))]
        for f in futures:
            f.result()
        return full_out

    def close(self) -> None:
        self._pool.shutdown(wait=True)
        for rt in self.runtimes:
            if rt is not None:
                rt.close()
        self.runtimes = []

    def __enter__(self) -> "ShardedRuntime":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


class RankGroup:
    """torch.distributed plumbing for one process per GPU (torchrun).

    Only the barrier around the timed region and the max-over-ranks of a
    timing cross ranks; the data path has no collective."""

    def __init__(self, world: int, rank: int, local_rank: int, backend: str | None) -> None:
        self.world, self.rank, self.local_rank, self.backend = world, rank, local_rank, backend

    @classmethod
    def from_env(cls, backend: str = "nccl", timeout_s: float = 300.0) -> "RankGroup":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        if world == 1:
            return cls(1, 0, local, None)
        import torch
        import torch.distributed as dist

        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
        return cls(world, rank, local, backend)

    def slice(self, batch: int) -> tuple[int, int]:
        return batch_slices(batch, self.world)[self.rank]

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def _reduce(self, value: float, op) -> float:
        if self.world == 1:
            return float(value)
        import torch
        import torch.distributed as dist

        dev = f"cuda:{self.local_rank}" if self.backend == "nccl" else "cpu"
        t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, value: float) -> float:
        import torch.distributed as dist

        return self._reduce(value, dist.ReduceOp.MAX) if self.world > 1 else float(value)

    def sum(self, value: float) -> float:
        import torch.distributed as dist

        return self._reduce(value, dist.ReduceOp.SUM) if self.world > 1 else float(value)

    def close(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()


__all__ = ["batch_slices", "ShardedRuntime", "RankGroup"]
