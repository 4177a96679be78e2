"""ctypes driver of the reference SPINNV2 runtime (oracle/_ref/libspkv2_ref.so).

TEST INFRASTRUCTURE: runs an SPK packaged for a CPU profile through the
reference's own load/prepare/set_input/run/get_output API
(reference runtime/include/spkv2_runtime.h:42-66).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

from . import REF_LIB

_lib = None


class FaultEventC(ctypes.Structure):
    """Spkv2FaultEvent (reference runtime/include/spkv2_runtime.h)."""
    _fields_ = [("node_id", ctypes.c_uint32), ("tensor_id", ctypes.c_uint32), ("element_index", ctypes.c_uint64),
                ("bit_index", ctypes.c_uint8), ("invocation_index", ctypes.c_uint32), ("seed", ctypes.c_uint64),
                ("enabled", ctypes.c_int)]


class StatsC(ctypes.Structure):
    """Spkv2ReliabilityStats."""
    _fields_ = [(n, ctypes.c_uint64) for n in ("injected_faults", "detected_faults", "recovered_faults",
                                                "unrecovered_faults", "rerun_count")]


class RangeObsC(ctypes.Structure):
    """Spkv2RangeObservation."""
    _fields_ = [("node_id", ctypes.c_uint32), ("tensor_id", ctypes.c_uint32), ("observed_min", ctypes.c_float),
                ("observed_max", ctypes.c_float), ("observations", ctypes.c_uint64)]


def library(path: str | Path | None = None) -> ctypes.CDLL:
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path or REF_LIB)
    if not p.exists():
        raise FileNotFoundError(f"{p} missing: build it with `make -C oracle ref`")
    lib = ctypes.CDLL(str(p))
    vp, sz, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    for name, res, args in [
        ("spkv2_load_memory", i32, [vp, sz, ctypes.POINTER(vp)]),
        ("spkv2_prepare", i32, [vp, vp, sz]),
        ("spkv2_set_input", i32, [vp, i32, vp, sz]),
        ("spkv2_get_output_size", i32, [vp, i32, ctypes.POINTER(sz)]),
        ("spkv2_get_output", i32, [vp, i32, vp, sz]),
        ("spkv2_run", i32, [vp]),
        ("spkv2_free", None, [vp]),
        ("spkv2_set_fault_event", i32, [vp, ctypes.POINTER(FaultEventC)]),
        ("spkv2_clear_fault_event", None, [vp]),
        ("spkv2_get_reliability_stats", i32, [vp, ctypes.POINTER(StatsC)]),
        ("spkv2_reset_reliability_stats", None, [vp]),
        ("spkv2_get_range_observation", i32, [vp, ctypes.c_uint32, ctypes.POINTER(RangeObsC)]),
        ("spkv2_reset_range_observations", None, [vp]),
    ]:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class RefRuntime:
    """One SPK on the reference CPU runtime (threads: OMP_NUM_THREADS)."""

    def __init__(self, spk: bytes, out_specs: list[tuple[tuple, type]]):
        self.lib = library()
        self._buf = ctypes.create_string_buffer(spk, len(spk))
        self.ctx = ctypes.c_void_p()
        rc = self.lib.spkv2_load_memory(self._buf, len(spk), ctypes.byref(self.ctx))
        if rc:
            raise RuntimeError(f"reference load failed: {rc}")
        rc = self.lib.spkv2_prepare(self.ctx, None, 0)
        if rc:
            raise RuntimeError(f"reference prepare failed: {rc}")
        self.out_specs = out_specs

    def run(self, *inputs: np.ndarray) -> list[np.ndarray]:
        for i, x in enumerate(inputs):
            a = np.ascontiguousarray(x)
            rc = self.lib.spkv2_set_input(self.ctx, i, a.ctypes.data, a.nbytes)
            if rc:
                raise RuntimeError(f"reference set_input failed: {rc}")
        rc = self.lib.spkv2_run(self.ctx)
        if rc:
            raise RuntimeError(f"reference run failed: {rc}")
        outs = []
        for i, (shape, dtype) in enumerate(self.out_specs):
            o = np.empty(shape, dtype=dtype)
            rc = self.lib.spkv2_get_output(self.ctx, i, o.ctypes.data, o.nbytes)
            if rc:
                raise RuntimeError(f"reference get_output failed: {rc}")
            outs.append(o)
        return outs

    def run_reliability(self, inputs: list[np.ndarray], event: dict | None, node_ids: list[int]):
        """One run with reset statistics and an optional fault event
        (dict of Spkv2FaultEvent fields); returns (outputs, stats dict,
        {node_id: (min, max, observations)} for the nodes observed)."""
        self.lib.spkv2_reset_reliability_stats(self.ctx)
        self.lib.spkv2_reset_range_observations(self.ctx)
        if event is None:
            self.lib.spkv2_clear_fault_event(self.ctx)
        else:
            ev = FaultEventC(**{**event, "enabled": 1})
            rc = self.lib.spkv2_set_fault_event(self.ctx, ctypes.byref(ev))
            if rc:
                raise RuntimeError(f"reference set_fault_event failed: {rc}")
        outs = self.run(*inputs)
        st = StatsC()
        self.lib.spkv2_get_reliability_stats(self.ctx, ctypes.byref(st))
        obs = {}
        for nid in node_ids:
            o = RangeObsC()
            if self.lib.spkv2_get_range_observation(self.ctx, nid, ctypes.byref(o)) == 0 and o.observations:
                obs[nid] = (float(o.observed_min), float(o.observed_max), int(o.observations))
        return outs, {n: int(getattr(st, n)) for n, _ in st._fields_}, obs

    def close(self):
        if self.ctx:
            self.lib.spkv2_free(self.ctx)
            self.ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def run_reference(spk: bytes, inputs: list[np.ndarray], out_specs) -> list[np.ndarray]:
    rt = RefRuntime(spk, out_specs)
    try:
        return rt.run(*inputs)
    finally:
        rt.close()


def threads() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
