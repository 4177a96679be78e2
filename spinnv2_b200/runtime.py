"""ctypes driver of libspkv2_runtime.so, the B200 CUDA target of the SPINNV2
runtime.

`RuntimeDriver` keeps the interface of SPINNV2's reliability driver
(reference research/reliability/runtime_driver.py:44-128: construct from a
library path and an SPK path, run(input, event) -> (output, stats),
range_observations, close), so scripts written against the CPU runtime work
unchanged when pointed at this library.  `Runtime` is the fuller wrapper
used by the tests and the benchmark: multiple inputs/outputs, host or device
bindings, asynchronous runs, per-tensor reads/writes and per-node variants.

The library is the product path: if it is missing, importing works but every
constructor raises; nothing here falls back to a CPU implementation.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .spk import SpkPackage, read_spk

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libspkv2_runtime.so"

MATH_SPEC, MATH_3XTF32, MATH_TF32, MATH_FP32 = 0, 1, 2, 3
LAYOUT_ROWMAJOR, LAYOUT_NHWC = 1, 2


class Spkv2Error(RuntimeError):
    def __init__(self, action: str, code: int, text: str = "") -> None:
        super().__init__(f"SPINNV2 runtime {action} failed with {code}" + (f" ({text})" if text else ""))
        self.code = code


class CSpkv2FaultEvent(ctypes.Structure):
    _fields_ = [
        ("node_id", ctypes.c_uint32),
        ("tensor_id", ctypes.c_uint32),
        ("element_index", ctypes.c_uint64),
        ("bit_index", ctypes.c_uint8),
        ("invocation_index", ctypes.c_uint32),
        ("seed", ctypes.c_uint64),
        ("enabled", ctypes.c_int),
    ]


class CSpkv2ReliabilityStats(ctypes.Structure):
    _fields_ = [
        ("injected_faults", ctypes.c_uint64),
        ("detected_faults", ctypes.c_uint64),
        ("recovered_faults", ctypes.c_uint64),
        ("unrecovered_faults", ctypes.c_uint64),
        ("rerun_count", ctypes.c_uint64),
    ]


class CSpkv2RangeObservation(ctypes.Structure):
    _fields_ = [
        ("node_id", ctypes.c_uint32),
        ("tensor_id", ctypes.c_uint32),
        ("observed_min", ctypes.c_float),
        ("observed_max", ctypes.c_float),
        ("observations", ctypes.c_uint64),
    ]


@dataclass
class FaultEvent:
    node_id: int
    tensor_id: int
    element_index: int
    bit_index: int
    invocation_index: int = 1
    seed: int = 0


_LIB = None


def load_library(path: str | Path | None = None) -> ctypes.CDLL:
    """Load (once) and type the runtime library; raises if it is not built."""
    global _LIB
    if path is None and _LIB is not None:
        return _LIB
    p = Path(path or os.environ.get("SPKV2_RUNTIME_LIB", LIB_PATH))
    if not p.exists():
        raise FileNotFoundError(f"{p} is not built; run __graft_entry__.build() or spinnv2_b200/csrc/build.py")
    lib = ctypes.CDLL(str(p))
    vp, sz, i32, u32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32
    sig = {
        "spkv2_runtime_version": (ctypes.c_char_p, []),
        "spkv2_load_file": (i32, [ctypes.c_char_p, ctypes.POINTER(vp)]),
        "spkv2_load_memory": (i32, [vp, sz, ctypes.POINTER(vp)]),
        "spkv2_prepare": (i32, [vp, vp, sz]),
        "spkv2_prepare_with_scratch": (i32, [vp, vp, sz, vp, sz]),
        "spkv2_set_input": (i32, [vp, i32, vp, sz]),
        "spkv2_bind_input": (i32, [vp, i32, vp, sz]),
        "spkv2_bind_output": (i32, [vp, i32, vp, sz]),
        "spkv2_get_output_size": (i32, [vp, i32, ctypes.POINTER(sz)]),
        "spkv2_get_output": (i32, [vp, i32, vp, sz]),
        "spkv2_run": (i32, [vp]),
        "spkv2_set_fault_event": (i32, [vp, ctypes.POINTER(CSpkv2FaultEvent)]),
        "spkv2_clear_fault_event": (None, [vp]),
        "spkv2_get_reliability_stats": (i32, [vp, ctypes.POINTER(CSpkv2ReliabilityStats)]),
        "spkv2_reset_reliability_stats": (None, [vp]),
        "spkv2_get_range_observation": (i32, [vp, u32, ctypes.POINTER(CSpkv2RangeObservation)]),
        "spkv2_reset_range_observations": (None, [vp]),
        "spkv2_profile_dump": (None, []),
        "spkv2_free": (None, [vp]),
        "spkv2_register_kernel": (i32, [ctypes.c_uint16, ctypes.c_uint16, ctypes.c_uint16, vp, i32]),
        "spkv2_clear_user_kernels": (None, []),
        "spkv2_cuda_set_device": (i32, [vp, i32]),
        "spkv2_cuda_get_device": (i32, [vp, ctypes.POINTER(i32)]),
        "spkv2_cuda_set_math_mode": (i32, [vp, i32]),
        "spkv2_cuda_set_graph_mode": (i32, [vp, i32]),
        "spkv2_cuda_stream": (vp, [vp]),
        "spkv2_cuda_tensor_device_ptr": (vp, [vp, u32]),
        "spkv2_cuda_tensor_layout": (i32, [vp, u32]),
        "spkv2_cuda_run_async": (i32, [vp]),
        "spkv2_cuda_synchronize": (i32, [vp]),
        "spkv2_cuda_run_nodes": (i32, [vp, u32, u32]),
        "spkv2_cuda_watchdog_probe": (i32, [vp, u32, ctypes.POINTER(i32)]),
        "spkv2_cuda_last_device_code": (i32, [vp]),
        "spkv2_cuda_profile_nodes": (i32, [vp, ctypes.POINTER(ctypes.c_float), u32]),
        "spkv2_cuda_read_tensor": (i32, [vp, u32, vp, sz]),
        "spkv2_cuda_write_tensor": (i32, [vp, u32, vp, sz]),
        "spkv2_cuda_launches_per_run": (i32, [vp, ctypes.POINTER(u32)]),
        "spkv2_cuda_node_variant": (ctypes.c_char_p, [vp, u32]),
        "spkv2_cuda_status_string": (ctypes.c_char_p, [i32]),
        "spkv2_fnv1a32": (u32, [vp, sz]),
        "spkv2_platform_set_device_allocator": (i32, [vp, vp, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


class Runtime:
    """One SPK model prepared on one B200."""

    def __init__(self, spk: str | Path | bytes, *, device: int | None = None, math_mode: int | None = None,
                 graph: bool = True, prepare: bool = True, lib: ctypes.CDLL | None = None) -> None:
        self.lib = lib or load_library()
        self._model = bytes(spk) if isinstance(spk, (bytes, bytearray)) else Path(spk).read_bytes()
        self._model_buf = ctypes.create_string_buffer(self._model, len(self._model))
        self.package: SpkPackage = read_spk(self._model)
        self.ctx = ctypes.c_void_p()
        self._check(self.lib.spkv2_load_memory(self._model_buf, len(self._model), ctypes.byref(self.ctx)), "load")
        self._keep: dict = {}
        if device is not None:
            self._check(self.lib.spkv2_cuda_set_device(self.ctx, int(device)), "set device")
        if math_mode is not None:
            self._check(self.lib.spkv2_cuda_set_math_mode(self.ctx, int(math_mode)), "set math mode")
        self._check(self.lib.spkv2_cuda_set_graph_mode(self.ctx, 1 if graph else 0), "set graph mode")
        if prepare:
            self.prepare()

    # -------------------------------------------------------------- basics
    def _check(self, code: int, action: str) -> None:
        if code != 0:
            text = self.lib.spkv2_cuda_status_string(code)
            raise Spkv2Error(action, code, text.decode() if text else "")

    def prepare(self, arena=None, arena_size: int = 0, scratch=None, scratch_size: int = 0) -> None:
        self._check(self.lib.spkv2_prepare_with_scratch(self.ctx, arena, arena_size, scratch, scratch_size),
                    "prepare")

    def close(self) -> None:
        if self.ctx:
            self.lib.spkv2_free(self.ctx)
            self.ctx = ctypes.c_void_p()

    def __enter__(self) -> "Runtime":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    # -------------------------------------------------------------- IO
    def _arr(self, tensor, value) -> np.ndarray:
        a = np.ascontiguousarray(value, dtype=tensor.np_dtype)
        if a.nbytes != tensor.size_bytes:
            raise ValueError(f"tensor {tensor.name}: expected {tensor.size_bytes} bytes, got {a.nbytes}")
        return a

    def set_input(self, index: int, value) -> None:
        a = self._arr(self.package.inputs[index], value)
        self._check(self.lib.spkv2_set_input(self.ctx, index, a.ctypes.data, a.nbytes), "set input")

    def bind_input(self, index: int, value) -> None:
        """Bind a host array (kept alive here) or a device pointer (int)."""
        t = self.package.inputs[index]
        if isinstance(value, int):
            self._check(self.lib.spkv2_bind_input(self.ctx, index, value, t.size_bytes), "bind input")
            return
        a = self._arr(t, value)
        self._keep[("in", index)] = a
        self._check(self.lib.spkv2_bind_input(self.ctx, index, a.ctypes.data, a.nbytes), "bind input")

    def bind_output(self, index: int, value) -> None:
        t = self.package.outputs[index]
        if isinstance(value, int):
            self._check(self.lib.spkv2_bind_output(self.ctx, index, value, t.size_bytes), "bind output")
            return
        if not (isinstance(value, np.ndarray) and value.flags.c_contiguous and value.nbytes == t.size_bytes):
            raise ValueError("bind_output needs a C-contiguous array of the output's size")
        self._keep[("out", index)] = value
        self._check(self.lib.spkv2_bind_output(self.ctx, index, value.ctypes.data, value.nbytes), "bind output")

    def get_output(self, index: int = 0) -> np.ndarray:
        t = self.package.outputs[index]
        out = np.empty(t.shape, dtype=t.np_dtype)
        self._check(self.lib.spkv2_get_output(self.ctx, index, out.ctypes.data, out.nbytes), "get output")
        return out

    def outputs(self) -> list[np.ndarray]:
        return [self.get_output(i) for i in range(len(self.package.outputs))]

    # -------------------------------------------------------------- execution
    def run(self, *inputs) -> list[np.ndarray] | None:
        for i, x in enumerate(inputs):
            self.set_input(i, x)
        self._check(self.lib.spkv2_run(self.ctx), "run")
        return self.outputs() if inputs else None

    def run_async(self) -> None:
        self._check(self.lib.spkv2_cuda_run_async(self.ctx), "run async")

    def synchronize(self) -> None:
        self._check(self.lib.spkv2_cuda_synchronize(self.ctx), "synchronize")

    def run_nodes(self, first: int, last: int) -> None:
        """Run nodes [first, last) eagerly on the current tensor contents.

        Inputs are not staged: the memory plan may reuse a graph input's
        buffer after its last reader, so call set_input() again before
        re-running nodes that read an input."""
        self._check(self.lib.spkv2_cuda_run_nodes(self.ctx, first, last), "run nodes")

    # -------------------------------------------------------------- introspection
    def read_tensor(self, tid: int) -> np.ndarray:
        t = self.package.tensors[tid]
        out = np.empty(t.shape, dtype=t.np_dtype)
        self._check(self.lib.spkv2_cuda_read_tensor(self.ctx, tid, out.ctypes.data, out.nbytes), "read tensor")
        return out

    def write_tensor(self, tid: int, value) -> None:
        a = self._arr(self.package.tensors[tid], value)
        self._check(self.lib.spkv2_cuda_write_tensor(self.ctx, tid, a.ctypes.data, a.nbytes), "write tensor")

    def tensor_layout(self, tid: int) -> int:
        return int(self.lib.spkv2_cuda_tensor_layout(self.ctx, tid))

    def node_variant(self, nid: int) -> str:
        v = self.lib.spkv2_cuda_node_variant(self.ctx, nid)
        return v.decode() if v else ""

    def launches_per_run(self) -> int:
        n = ctypes.c_uint32()
        self._check(self.lib.spkv2_cuda_launches_per_run(self.ctx, ctypes.byref(n)), "launch count")
        return int(n.value)

    def profile_nodes(self) -> np.ndarray:
        """Device milliseconds of every node from one eager, event-bracketed run."""
        n = len(self.package.nodes)
        out = (ctypes.c_float * max(n, 1))()
        self._check(self.lib.spkv2_cuda_profile_nodes(self.ctx, out, n), "profile nodes")
        return np.array(out[:n], dtype=np.float64)

    def watchdog_probe(self, wait_us: int = 1000) -> tuple[int, int]:
        """Run the bounded-wait self-test; returns (return code, recorded code)."""
        code = ctypes.c_int(0)
        rc = self.lib.spkv2_cuda_watchdog_probe(self.ctx, int(wait_us), ctypes.byref(code))
        return int(rc), int(code.value)

    def stream(self) -> int:
        return int(self.lib.spkv2_cuda_stream(self.ctx) or 0)

    def device_ptr(self, tid: int) -> int:
        return int(self.lib.spkv2_cuda_tensor_device_ptr(self.ctx, tid) or 0)


class RuntimeDriver:
    """Drop-in for the reference reliability driver: fp32 input 0 -> output 0."""

    def __init__(self, library_path: str | Path, spk_path: str | Path) -> None:
        self.rt = Runtime(spk_path, lib=load_library(library_path))
        self.lib = self.rt.lib
        self.ctx = self.rt.ctx

    def close(self) -> None:
        self.rt.close()

    def __enter__(self) -> "RuntimeDriver":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def run(self, input_data: np.ndarray, event: FaultEvent | None = None) -> tuple[np.ndarray, dict]:
        values = np.ascontiguousarray(input_data, dtype=np.float32)
        self.rt._check(self.lib.spkv2_set_input(self.ctx, 0, values.ctypes.data, values.nbytes), "set input")
        self.lib.spkv2_reset_reliability_stats(self.ctx)
        self.lib.spkv2_reset_range_observations(self.ctx)
        if event is None:
            self.lib.spkv2_clear_fault_event(self.ctx)
        else:
            ev = CSpkv2FaultEvent(event.node_id, event.tensor_id, event.element_index, event.bit_index,
                                  event.invocation_index, event.seed, 1)
            self.rt._check(self.lib.spkv2_set_fault_event(self.ctx, ctypes.byref(ev)), "set event")
        self.rt._check(self.lib.spkv2_run(self.ctx), "run")
        size = ctypes.c_size_t()
        self.rt._check(self.lib.spkv2_get_output_size(self.ctx, 0, ctypes.byref(size)), "output size")
        out = np.empty(size.value // 4, dtype=np.float32)
        self.rt._check(self.lib.spkv2_get_output(self.ctx, 0, out.ctypes.data, out.nbytes), "get output")
        stats = CSpkv2ReliabilityStats()
        self.rt._check(self.lib.spkv2_get_reliability_stats(self.ctx, ctypes.byref(stats)), "stats")
        return out, {name: int(getattr(stats, name)) for name, _ in stats._fields_}

    def range_observations(self, node_ids: list[int]) -> list[dict]:
        recs = []
        for nid in node_ids:
            ob = CSpkv2RangeObservation()
            self.rt._check(self.lib.spkv2_get_range_observation(self.ctx, nid, ctypes.byref(ob)), "range")
            if ob.observations:
                recs.append({"node_id": int(ob.node_id), "tensor_id": int(ob.tensor_id),
                             "observed_min": float(ob.observed_min), "observed_max": float(ob.observed_max),
                             "observations": int(ob.observations)})
        return recs
