"""The C-ABI library on the CPU: it loads without a GPU, exports every function
the headers declare, and keeps the reference's loader and registry return
codes (reference runtime/core/loader.c:140-207, kernels/reference/kernels.c:
18-30, runtime/tests/test_register_kernel.c:134-148)."""

from __future__ import annotations

import ctypes
import re
import struct
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _declared_functions() -> set[str]:
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(spkv2_\w+)\s*\(", text, flags=re.M))
    return names


def test_library_exports_every_declared_function(built):
    from spinnv2_b200.runtime import LIB_PATH

    lib = ctypes.CDLL(str(LIB_PATH))
    declared = _declared_functions()
    assert len(declared) >= 55
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_registry_return_codes(built):
    from spinnv2_b200.runtime import load_library

    lib = load_library()
    CB = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p)
    noop = CB(lambda *a: 0)
    lib.spkv2_clear_user_kernels()
    assert lib.spkv2_register_kernel(6, 1, 1, None, 1) == -1
    for i in range(64):
        assert lib.spkv2_register_kernel(200 + i, 1, 1, ctypes.cast(noop, ctypes.c_void_p), 1) == 0
    assert lib.spkv2_register_kernel(999, 1, 1, ctypes.cast(noop, ctypes.c_void_p), 1) == -2
    lib.spkv2_clear_user_kernels()
    assert lib.spkv2_register_kernel(999, 1, 1, ctypes.cast(noop, ctypes.c_void_p), 1) == 0
    lib.spkv2_clear_user_kernels()


def _load(lib, data: bytes) -> int:
    buf = ctypes.create_string_buffer(data, len(data))
    ctx = ctypes.c_void_p()
    rc = lib.spkv2_load_memory(buf, len(data), ctypes.byref(ctx))
    if rc == 0:
        lib.spkv2_free(ctx)
    return rc


def test_loader_error_codes(built):
    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import load_library

    lib = load_library()
    spk = bytearray(pipeline.compile_config("lenet5", 1, targets=("cuda_b200",))["cuda_b200"])
    assert _load(lib, bytes(spk)) == 0
    bad_magic = bytearray(spk)
    bad_magic[0] ^= 0xFF
    assert _load(lib, bytes(bad_magic)) == -2
    corrupt = bytearray(spk)
    corrupt[len(corrupt) // 2] ^= 0x01  # inside the weights
    assert _load(lib, bytes(corrupt)) == -6
    bad_dir = bytearray(spk)
    struct.pack_into("<I", bad_dir, 12, 100000)  # section_count far past the file
    assert _load(lib, bytes(bad_dir)) == -3
    assert _load(lib, bytes(spk[:40])) == -1


def test_fnv_helper_matches_python(built):
    from spinnv2_b200.compiler.spk_writer import fnv1a32
    from spinnv2_b200.runtime import load_library

    lib = load_library()
    data = bytes(range(256)) * 300
    assert lib.spkv2_fnv1a32(data[:4096], 4096) == fnv1a32(data[:4096])
    h = 0x811C9DC5
    for b in data:
        h = ((h ^ b) * 0x01000193) & 0xFFFFFFFF
    assert lib.spkv2_fnv1a32(data, len(data)) == h


def test_prepare_without_a_device_fails_cleanly(built):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from spinnv2_b200.compiler import pipeline
    from spinnv2_b200.runtime import Runtime, Spkv2Error

    spk = pipeline.compile_config("lenet5", 1, targets=("cuda_b200",))["cuda_b200"]
    with pytest.raises(Spkv2Error) as e:
        Runtime(spk)
    assert e.value.code == -42
