"""qwowl35_b200 -- Qwen3.5-9B decode hot path for NVIDIA B200 (sm_100a).

The product is libqw35cuda.so (C ABI in include/qw35_ffi.h and
include/qw35_cuda.h).  This package holds its sources (csrc/), the in-tree
build (build.py), a ctypes binding (_lib.py), the host-side mirror of the
reference's runtime wrapper (runtime.py), torch-tensor helpers for the per-op
entry points (ops.py) and the synthetic cooked-GGUF model generator (synth.py).
"""
from ._lib import LIB_PATH, Qw35Error, header_symbols, lib

__all__ = ["LIB_PATH", "Qw35Error", "header_symbols", "lib"]
