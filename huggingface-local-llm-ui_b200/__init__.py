"""B200-native GGUF dequant-GEMV decode path (host side).

The compute lives in libb2q.so (csrc/, CUDA for sm_100a behind the C ABI
declared in include/b2q.h).  This package is the Python mirror of the
reference's GPU-engine and model interfaces over that ABI, plus the
synthetic-GGUF generator the benchmarks use.
"""
from . import ggml, synth  # noqa: F401
