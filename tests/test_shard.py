"""Batch-sharded multi-GPU path: slicing, the single-process multi-device
driver (with a CPU stand-in runtime), and the one-process-per-rank plumbing
over world_size-2 gloo process groups.  The data path has no collective; the
gloo tests check the barrier / max-over-ranks used around the timed region
and that the per-rank slices reassemble the full batch."""

from __future__ import annotations

import ctypes
import multiprocessing as mp
import os
import socket
import time
from types import SimpleNamespace

import numpy as np
import pytest

from conftest import compile_pair, reference_outputs, seeded_input


def test_batch_slices_cover_the_batch_contiguously():
    from spinnv2_b200.shard import batch_slices

    for batch in (0, 1, 5, 8, 63, 64, 256):
        for world in (1, 2, 3, 4, 8):
            sl = batch_slices(batch, world)
            assert len(sl) == world
            per = -(-batch // world) if batch else 0
            pos = 0
            for start, count in sl:
                assert start == min(pos, batch)
                assert 0 <= count <= per
                pos += count
            assert pos == batch
    assert batch_slices(64, 8) == [(8 * r, 8) for r in range(8)]
    assert batch_slices(5, 2) == [(0, 3), (3, 2)]
    assert batch_slices(2, 4) == [(0, 1), (1, 1), (2, 0), (2, 0)]
    with pytest.raises(ValueError):
        batch_slices(4, 0)


# ---------------------------------------------------------------- stand-in runtime


def _stand_in(x: np.ndarray) -> np.ndarray:
    """Per-image function the fake runtime computes: row sums and squares."""
    flat = x.reshape(x.shape[0], -1).astype(np.float32)
    return np.stack([flat.sum(axis=1), (flat * flat).sum(axis=1)], axis=1)


class _FakeLib:
    def __init__(self, rt):
        self.rt = rt

    def spkv2_run(self, ctx):
        rt = self.rt
        n = rt.batch
        xin = np.ctypeslib.as_array(ctypes.cast(rt.bound_in, ctypes.POINTER(ctypes.c_float)), (n, 3, 4))
        out = np.ctypeslib.as_array(ctypes.cast(rt.bound_out, ctypes.POINTER(ctypes.c_float)), (n, 2))
        time.sleep(0.01)  # let the device threads overlap
        out[...] = _stand_in(xin)
        rt.runs += 1
        return 0


class _FakeRuntime:
    """Implements the slice of `Runtime` that ShardedRuntime uses."""

    made: list = []

    def __init__(self, spk, device=None, math_mode=None, graph=True):
        self.batch = int(spk.decode().split("=")[1])
        self.device = device
        t_in = SimpleNamespace(name="x", shape=(self.batch, 3, 4), np_dtype=np.float32)
        t_out = SimpleNamespace(name="y", shape=(self.batch, 2), np_dtype=np.float32)
        self.package = SimpleNamespace(inputs=[t_in], outputs=[t_out])
        self.lib = _FakeLib(self)
        self.ctx = object()
        self.runs = 0
        self.closed = False
        _FakeRuntime.made.append(self)

    def bind_input(self, k, ptr):
        self.bound_in = ptr

    def bind_output(self, k, ptr):
        self.bound_out = ptr

    def _check(self, code, what):
        assert code == 0, what

    def close(self):
        self.closed = True


def test_sharded_runtime_places_each_slice_at_its_offset():
    from spinnv2_b200.shard import ShardedRuntime

    _FakeRuntime.made = []
    asked = []

    def spk_for(n):
        asked.append(n)
        return f"n={n}".encode()

    x = seeded_input((7, 3, 4))
    with ShardedRuntime(spk_for, 7, [0, 1, 2], runtime_factory=_FakeRuntime) as sr:
        assert sr.slices == [(0, 3), (3, 3), (6, 1)]
        assert sorted(asked) == [1, 3]  # one package per distinct slice size
        assert [rt.device for rt in _FakeRuntime.made] == [0, 1, 2]
        for _ in range(2):
            (y,) = sr.run(x)
            np.testing.assert_array_equal(y, _stand_in(x))
        with pytest.raises(ValueError):
            sr.run(x[:6])
    assert all(rt.closed and rt.runs == 2 for rt in _FakeRuntime.made)


def test_sharded_runtime_with_idle_ranks():
    from spinnv2_b200.shard import ShardedRuntime

    _FakeRuntime.made = []
    x = seeded_input((2, 3, 4), seed=3)
    with ShardedRuntime(lambda n: f"n={n}".encode(), 2, [0, 1, 2, 3], runtime_factory=_FakeRuntime) as sr:
        assert len(_FakeRuntime.made) == 2
        (y,) = sr.run(x)
    np.testing.assert_array_equal(y, _stand_in(x))


# ---------------------------------------------------------------- gloo ranks


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_env(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))


def _gloo_worker(rank: int, world: int, port: int, batch: int, q) -> None:
    _rank_env(rank, world, port)
    import torch.distributed as dist

    from spinnv2_b200.shard import RankGroup

    g = RankGroup.from_env(backend="gloo", timeout_s=60)
    try:
        start, count = g.slice(batch)
        x = seeded_input((batch, 3, 4), seed=5)
        y_local = _stand_in(x[start:start + count])
        g.barrier()
        t_max = g.max(0.5 * (rank + 1))
        n_sum = g.sum(float(count))
        gathered = [None] * world
        dist.all_gather_object(gathered, (start, y_local))
        q.put((rank, t_max, n_sum, gathered))
    finally:
        g.close()


def _run_ranks(target, world: int, *args, timeout: float = 120.0) -> list:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.time() + timeout
    try:
        for _ in range(world):
            results.append(q.get(timeout=max(1.0, deadline - time.time())))
    finally:
        for p in procs:
            p.join(timeout=max(1.0, deadline - time.time()))
            if p.is_alive():
                p.kill()
    return sorted(results, key=lambda r: r[0])


def test_two_gloo_ranks_shard_the_batch_and_agree_on_timing():
    batch = 9
    res = _run_ranks(_gloo_worker, 2, batch)
    assert [r[0] for r in res] == [0, 1]
    for rank, t_max, n_sum, gathered in res:
        assert t_max == 1.0  # max over ranks of 0.5 * (rank + 1)
        assert n_sum == batch
        y = np.concatenate([yl for _, yl in sorted(gathered, key=lambda g: g[0])])
        np.testing.assert_array_equal(y, _stand_in(seeded_input((batch, 3, 4), seed=5)))


def _put_and_exit(q, item) -> None:
    q.put(item)
    q.close()
    q.join_thread()  # flush the queue's feeder thread before the hard exit
    os._exit(0)


def _dropout_worker(rank: int, world: int, port: int, q) -> None:
    """Both ranks pass one barrier; then rank 1 leaves and never reaches the
    second.  Rank 0 must get an error from that barrier, not wait forever."""
    _rank_env(rank, world, port)
    from spinnv2_b200.shard import RankGroup

    try:
        g = RankGroup.from_env(backend="gloo", timeout_s=5)
        g.barrier()
    except Exception as e:  # noqa: BLE001
        _put_and_exit(q, (rank, f"setup failed: {type(e).__name__}: {e}"))
    if rank == 1:
        _put_and_exit(q, (1, "left"))
    t0 = time.time()
    try:
        g.barrier()
        item = (0, "barrier returned")
    except Exception as e:  # noqa: BLE001 - any error ends the wait
        item = (0, f"error after {time.time() - t0:.1f}s: {type(e).__name__}")
    _put_and_exit(q, item)


def test_a_rank_that_leaves_ends_the_other_ranks_barrier_with_an_error():
    res = _run_ranks(_dropout_worker, 2, timeout=90.0)
    assert res[1][1] == "left"
    assert res[0][1].startswith("error after"), res[0][1]


# ---------------------------------------------------------------- on the GPU


@pytest.mark.gpu
def test_sharded_lenet_on_two_contexts_matches_reference(gpu):
    """Two replicas (both on cuda:0 when one GPU is visible) serve slices 3+2
    of a batch of 5; the stitched outputs equal the reference runtime's
    output for the whole batch."""
    import torch

    from spinnv2_b200.shard import ShardedRuntime

    devices = [0, 1] if torch.cuda.device_count() > 1 else [0, 0]
    x = seeded_input((5, 1, 28, 28), "uniform", seed=2)
    ref = reference_outputs(compile_pair("lenet5", 5, targets=("cpu_generic_x86",))["cpu_generic_x86"], [x])[0]
    with ShardedRuntime(lambda n: compile_pair("lenet5", n, targets=("cuda_b200",))["cuda_b200"], 5, devices) as sr:
        assert sr.slices == [(0, 3), (3, 2)]
        for _ in range(3):
            (y,) = sr.run(x)
            np.testing.assert_allclose(y, ref, atol=1e-3, rtol=1e-4)
