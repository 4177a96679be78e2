"""Target profiles: lookup and checking against the profile schema.

A profile is a JSON object with the fields the SPINNV2 target-profile schema
lists (reference compiler/target/target_profile.schema.json): name, word size
(32 or 64), endianness, alignment, memory caps, features, layouts, backends
and, per op, an ordered list of kernel tokens.  `check_profile` walks a field
table derived from that schema and reports every violation at once.

Bundled profiles (spinnv2_b200/compiler/profiles/*.json):

  cuda_b200        the B200 CUDA target (backend `delegate`, NHWC activations,
                   no `ref` token so no CPU fallback spec is ever emitted,
                   HBM-sized arena caps, 256-byte tensor alignment)
  cpu_generic_x86  the reference's cpu_generic token lists with the Apple-only
                   BNNS conv token removed and the arena caps raised, used to
                   package the CPU baseline the reference runtime times
  cpu_ref_large    scalar reference kernels only (strict CPU oracle)

The CUDA profile adds two optional fields: "memory_plan" (booleans) switches
off the planner's aliases whose meaning depends on NCHW byte order, and
"weight_layouts" lists the weight layouts its packages may store ("OIHW",
"TC_PANEL_F32X2": tensor-core convs' weights pre-packed by the SPK writer).
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Callable

BUNDLED = Path(__file__).resolve().parent / "profiles"


def _is_int(v: Any) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _str_list(v: Any) -> bool:
    return isinstance(v, list) and all(isinstance(x, str) for x in v)


# field -> (required, predicate, what the predicate demands)
_Rule = tuple[bool, Callable[[Any], bool], str]
TOP_FIELDS: dict[str, _Rule] = {
    "name": (True, lambda v: isinstance(v, str), "a string"),
    "word_size": (True, lambda v: _is_int(v) and v in (32, 64), "32 or 64"),
    "endianness": (True, lambda v: v in ("little", "big"), '"little" or "big"'),
    "alignment": (True, lambda v: _is_int(v) and v >= 1, "an integer >= 1"),
    "memory": (True, lambda v: isinstance(v, dict), "an object"),
    "features": (True, _str_list, "a list of strings"),
    "layouts": (True, _str_list, "a list of strings"),
    "backends": (True, _str_list, "a list of strings"),
    "ops": (True, lambda v: isinstance(v, dict) and all(_str_list(t) for t in v.values()),
            "an object mapping op names to lists of kernel tokens"),
    "memory_plan": (False, lambda v: isinstance(v, dict) and all(isinstance(x, bool) for x in v.values()),
                    "an object of booleans"),
    "weight_layouts": (False, lambda v: _str_list(v) and set(v) <= {"OIHW", "TC_PANEL_F32X2"},
                       'a list of weight layouts ("OIHW", "TC_PANEL_F32X2")'),
}
MEMORY_FIELDS: dict[str, _Rule] = {
    "activation_arena_max": (True, lambda v: _is_int(v) and v >= 0, "an integer >= 0"),
    "scratch_arena_max": (True, lambda v: _is_int(v) and v >= 0, "an integer >= 0"),
    "allow_runtime_malloc": (True, lambda v: isinstance(v, bool), "a boolean"),
}


def _violations(obj: dict[str, Any], rules: dict[str, _Rule], where: str) -> list[str]:
    out = []
    for key, (required, ok, demand) in rules.items():
        if key not in obj:
            if required:
                out.append(f"{where}{key}: required field is absent")
        elif not ok(obj[key]):
            out.append(f"{where}{key}: must be {demand}, got {obj[key]!r}")
    return out


def check_profile(profile: Any) -> None:
    """Raise ValueError naming every field of `profile` that breaks the schema."""
    if not isinstance(profile, dict):
        raise ValueError("invalid target profile: the top level must be a JSON object")
    problems = _violations(profile, TOP_FIELDS, "")
    if isinstance(profile.get("memory"), dict):
        problems += _violations(profile["memory"], MEMORY_FIELDS, "memory.")
    if problems:
        raise ValueError(f"invalid target profile {profile.get('name', '?')!r}: " + "; ".join(problems))


def load_target_profile(name_or_path: str | Path) -> dict[str, Any]:
    """A bundled profile by name, or a profile file by path, checked."""
    candidates = [Path(name_or_path), BUNDLED / f"{name_or_path}.json"]
    path = next((c for c in candidates if c.is_file()), None)
    if path is None:
        raise FileNotFoundError(f"no target profile named or at {name_or_path!s}")
    profile = json.loads(path.read_text(encoding="utf-8"))
    check_profile(profile)
    return profile


def is_cuda_profile(profile: dict[str, Any]) -> bool:
    """True for profiles that run on the CUDA target (backend `delegate`)."""
    return "delegate" in profile.get("backends", [])
