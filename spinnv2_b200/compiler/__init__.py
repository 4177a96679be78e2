"""Compiler side of the CUDA target: SIR -> passes -> kernel specs -> memory
plan -> SPK, plus the INT8 quantiser and the benchmark graph builders."""
