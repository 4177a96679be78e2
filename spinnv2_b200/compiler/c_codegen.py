"""Static C deployment wrapper for an SPK package.

Same public surface as the reference compiler's generated C (reference
compiler/codegen/c_codegen.py:180-325): a header with the package's size
macros (`<SYM>_INPUT_SIZE_i`, `<SYM>_OUTPUT_SIZE_i`, counts, arena sizes,
`<SYM>_SPK_CHECKSUM`; added here: `<SYM>_INPUT_SIZES` / `<SYM>_OUTPUT_SIZES`,
array initialisers for <sym>_run_multi) and a source that embeds the package
bytes and exports

    int  <sym>_init(void);
    int  <sym>_run(const void *input, void *output);
    int  <sym>_run_checked(const void *input, size_t input_size, void *output, size_t output_size);
    int  <sym>_run_multi(const void *const *inputs, const size_t *input_sizes, int num_inputs,
                         void *const *outputs, const size_t *output_sizes, int num_outputs);
    int  <sym>_verify_checksum(const void *data, size_t size);
    void <sym>_free(void);

with the reference's return codes (-1 null argument, -2 size mismatch or
checksum mismatch from verify, -10 embedded package checksum mismatch at
init, else the runtime's code).  The calling sequence is the runtime's
public API only: spkv2_load_memory (the embedded bytes are borrowed),
spkv2_prepare_with_scratch, spkv2_bind_input / spkv2_bind_output with the
caller's host buffers, spkv2_run, spkv2_free.  So one generated file links
against either runtime library: the reference CPU runtime or the CUDA
target's libspkv2_runtime.

Arenas.  For a CPU-profile package the wrapper reserves static host arenas
of the planned sizes, as the reference does.  For a `cuda_b200` package the
arenas live in device memory, owned by the runtime (it allocates them at
prepare from the package header), so the wrapper passes NULL / 0 and
reserves no host arena; inputs and outputs stay caller host buffers that
spkv2_run stages to and from the device.

Only the embedded-package mode is generated; the reference's external-
weights and inline (direct kernel call) modes are not.
"""

from __future__ import annotations

import re
from pathlib import Path

from ..spk import read_spk

_ROW = 16  # bytes per line of the embedded array


def _fnv1a32(data: bytes) -> int:
    h = 0x811C9DC5
    for b in data:
        h = ((h ^ b) * 0x01000193) & 0xFFFFFFFF
    return h


def _fnv1a32_fast(data: bytes) -> int:
    try:
        from ..runtime import load_library

        lib = load_library()
        return int(lib.spkv2_fnv1a32(data, len(data)))
    except Exception:  # noqa: BLE001 - library not built: the pure-Python hash
        return _fnv1a32(data)


def _check_symbol(symbol: str) -> None:
    if not re.fullmatch(r"[A-Za-z_][A-Za-z0-9_]*", symbol):
        raise ValueError(f"not a C identifier: {symbol!r}")


def _array_literal(data: bytes) -> str:
    rows = []
    for i in range(0, len(data), _ROW):
        rows.append("  " + ",".join(f"0x{b:02x}" for b in data[i:i + _ROW]) + ",")
    return "\n".join(rows)


def header_text(symbol: str, spk: bytes) -> str:
    _check_symbol(symbol)
    pkg = read_spk(spk)
    sym = symbol.upper()
    device = pkg.profile.get("name") == "cuda_b200"
    act = 0 if device else max(int(pkg.header["activation_arena_bytes"]), 1)
    scr = 0 if device else max(int(pkg.header["scratch_arena_bytes"]), 1)
    lines = [f"#ifndef {sym}_H", f"#define {sym}_H", "", "#include <stddef.h>", "",
             "#ifdef __cplusplus", 'extern "C" {', "#endif", ""]
    for i, t in enumerate(pkg.inputs):
        lines.append(f"#define {sym}_INPUT_SIZE_{i} ((size_t){int(t.size_bytes)}u)")
    for i, t in enumerate(pkg.outputs):
        lines.append(f"#define {sym}_OUTPUT_SIZE_{i} ((size_t){int(t.size_bytes)}u)")
    lines += [
        f"#define {sym}_INPUT_COUNT {len(pkg.inputs)}",
        f"#define {sym}_OUTPUT_COUNT {len(pkg.outputs)}",
        f"#define {sym}_INPUT_SIZE {sym}_INPUT_SIZE_0",
        f"#define {sym}_OUTPUT_SIZE {sym}_OUTPUT_SIZE_0",
        "/* All sizes, as array initialisers (an addition to the reference's macros). */",
        f"#define {sym}_INPUT_SIZES {{" + ", ".join(f"{sym}_INPUT_SIZE_{i}" for i in range(len(pkg.inputs))) + "}",
        f"#define {sym}_OUTPUT_SIZES {{" + ", ".join(f"{sym}_OUTPUT_SIZE_{i}" for i in range(len(pkg.outputs))) + "}",
        f"/* Host arena bytes the wrapper reserves (0: the runtime owns device arenas). */",
        f"#define {sym}_HOST_ARENAS {0 if device else 1}",
        f"#define {sym}_ACTIVATION_ARENA_SIZE ((size_t){act}u)",
        f"#define {sym}_SCRATCH_ARENA_SIZE ((size_t){scr}u)",
        f"#define {sym}_SPK_CHECKSUM 0x{_fnv1a32_fast(spk):08x}u",
        "",
        f"int {symbol}_init(void);",
        f"int {symbol}_run(const void *input, void *output);",
        f"int {symbol}_run_checked(const void *input, size_t input_size, void *output, size_t output_size);",
        f"int {symbol}_run_multi(const void *const *inputs, const size_t *input_sizes, int num_inputs,",
        f"    void *const *outputs, const size_t *output_sizes, int num_outputs);",
        f"int {symbol}_verify_checksum(const void *data, size_t size);",
        f"void {symbol}_free(void);",
        "",
        "#ifdef __cplusplus",
        "}",
        "#endif",
        "",
        f"#endif /* {sym}_H */",
        "",
    ]
    return "\n".join(lines)


def source_text(symbol: str, spk: bytes) -> str:
    _check_symbol(symbol)
    sym = symbol.upper()
    s = symbol
    return f"""/* Generated by spinnv2_b200.compiler.c_codegen: package {len(spk)} bytes. */
#include "{s}.h"

#include <stdint.h>

#include "spkv2_runtime.h"

/* 16-byte alignment lets the runtime read the package records in place. */
static const unsigned char {s}_spk[] __attribute__((aligned(16))) = {{
{_array_literal(spk)}
}};

#if {sym}_HOST_ARENAS
static unsigned char {s}_activation_arena[{sym}_ACTIVATION_ARENA_SIZE] __attribute__((aligned(64)));
static unsigned char {s}_scratch_arena[{sym}_SCRATCH_ARENA_SIZE] __attribute__((aligned(64)));
#define {sym}_ARENA {s}_activation_arena
#define {sym}_SCRATCH {s}_scratch_arena
#else
#define {sym}_ARENA ((void *)0)
#define {sym}_SCRATCH ((void *)0)
#endif

static Spkv2Context *{s}_ctx;

int {s}_verify_checksum(const void *data, size_t size) {{
    const unsigned char *p = (const unsigned char *)data;
    uint32_t h = 2166136261u;
    size_t i;
    if (!data || size == 0) return -1;
    for (i = 0; i < size; ++i) {{
        h ^= p[i];
        h *= 16777619u;
    }}
    return h == {sym}_SPK_CHECKSUM ? 0 : -2;
}}

int {s}_init(void) {{
    int rc;
    if ({s}_ctx) return 0;
    if ({s}_verify_checksum({s}_spk, sizeof({s}_spk)) != 0) return -10;
    rc = spkv2_load_memory({s}_spk, sizeof({s}_spk), &{s}_ctx);
    if (rc != 0) return rc;
    rc = spkv2_prepare_with_scratch({s}_ctx, {sym}_ARENA, {sym}_ACTIVATION_ARENA_SIZE,
                                    {sym}_SCRATCH, {sym}_SCRATCH_ARENA_SIZE);
    if (rc != 0) {{
        spkv2_free({s}_ctx);
        {s}_ctx = 0;
    }}
    return rc;
}}

int {s}_run_checked(const void *input, size_t input_size, void *output, size_t output_size) {{
    int rc;
    if (!input || !output) return -1;
    if (input_size != {sym}_INPUT_SIZE || output_size != {sym}_OUTPUT_SIZE) return -2;
    if ((rc = {s}_init()) != 0) return rc;
    if ((rc = spkv2_bind_input({s}_ctx, 0, (void *)input, input_size)) != 0) return rc;
    if ((rc = spkv2_bind_output({s}_ctx, 0, output, output_size)) != 0) return rc;
    return spkv2_run({s}_ctx);
}}

int {s}_run(const void *input, void *output) {{
    return {s}_run_checked(input, {sym}_INPUT_SIZE, output, {sym}_OUTPUT_SIZE);
}}

int {s}_run_multi(const void *const *inputs, const size_t *input_sizes, int num_inputs,
                  void *const *outputs, const size_t *output_sizes, int num_outputs) {{
    int rc, i;
    if (!inputs || !outputs || !input_sizes || !output_sizes) return -1;
    if ((rc = {s}_init()) != 0) return rc;
    for (i = 0; i < num_inputs; ++i)
        if ((rc = spkv2_bind_input({s}_ctx, i, (void *)inputs[i], input_sizes[i])) != 0) return rc;
    for (i = 0; i < num_outputs; ++i)
        if ((rc = spkv2_bind_output({s}_ctx, i, outputs[i], output_sizes[i])) != 0) return rc;
    return spkv2_run({s}_ctx);
}}

void {s}_free(void) {{
    spkv2_free({s}_ctx);
    {s}_ctx = 0;
}}
"""


def generate(spk: bytes, symbol: str, out_dir: str | Path) -> tuple[Path, Path]:
    """Write <symbol>.h and <symbol>.c for package `spk` into out_dir."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    h = out / f"{symbol}.h"
    c = out / f"{symbol}.c"
    h.write_text(header_text(symbol, spk))
    c.write_text(source_text(symbol, spk))
    return h, c
