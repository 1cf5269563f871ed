"""B200-native (sm_100a) routed-MoE hot path of Nebula, behind qwen/gpu.h's C ABI.

The product is the shared library ``libqwen_gpu.so`` built from ``csrc/``;
``lib`` is its ctypes binding (the same binding style as the reference's own
tests), ``build`` compiles it.
"""
from . import lib  # noqa: F401
