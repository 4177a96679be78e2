"""Target profiles: loading and validation.

Same profile schema as SPINNV2 (reference compiler/target/profile.py:10-55,
compiler/target/target_profile.schema.json): name, word size, endianness,
alignment, memory caps, features, layouts, backends and an ordered list of
kernel tokens per op.  Bundled profiles:

  cuda_b200        the B200 CUDA target (backend `delegate`, NHWC activations,
                   no `ref` token so no CPU fallback spec is ever emitted,
                   HBM-sized arena caps, 256-byte tensor alignment)
  cpu_generic_x86  the reference's cpu_generic token lists with the Apple-only
                   BNNS conv token removed and the arena caps raised, used to
                   package the CPU baseline the reference runtime times
  cpu_ref_large    scalar reference kernels only (strict CPU oracle)

The CUDA profile adds an optional "memory_plan" object that switches off the
planner's aliases whose meaning depends on NCHW byte order.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

REQUIRED_KEYS = {"name", "word_size", "endianness", "alignment", "memory", "features", "layouts", "backends", "ops"}


def profiles_dir() -> Path:
    return Path(__file__).resolve().parent / "profiles"


def load_target_profile(name_or_path: str) -> dict[str, Any]:
    path = Path(name_or_path)
    if not path.exists():
        path = profiles_dir() / f"{name_or_path}.json"
    if not path.exists():
        raise FileNotFoundError(f"target profile not found: {name_or_path}")
    profile = json.loads(path.read_text(encoding="utf-8"))
    validate_target_profile(profile)
    return profile


def validate_target_profile(profile: dict[str, Any]) -> None:
    missing = sorted(REQUIRED_KEYS - set(profile))
    if missing:
        raise ValueError(f"target profile missing keys: {', '.join(missing)}")
    if profile["endianness"] not in ("little", "big"):
        raise ValueError("target profile endianness must be 'little' or 'big'")
    for key in ("activation_arena_max", "scratch_arena_max", "allow_runtime_malloc"):
        if key not in profile["memory"]:
            raise ValueError(f"target profile memory missing key: {key}")
    if not isinstance(profile["ops"], dict):
        raise ValueError("target profile ops must be an object")


def is_cuda_profile(profile: dict[str, Any]) -> bool:
    return "delegate" in profile.get("backends", [])
