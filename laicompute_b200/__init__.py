"""B200-native engine for LAICompute's per-token Llama decode loop.

The compute path is the native library laicompute_b200/lib/liblaic_b200.so
(hand-written sm_100a kernels behind the C ABI of include/laic_b200.h).
This package holds its build recipe, a ctypes binding, the GGUF reader/writer
and the synthetic-model generator used by the tests and the benchmark.
"""
from . import gguf, synth  # noqa: F401

__all__ = ["gguf", "synth"]
