"""rosevine_b200: a B200-native (sm_100a) MoE-layer backend for Rosevine.

The product is librvcuda.so (C ABI, include/rvcuda.h) built from rosevine_b200/csrc by
rosevine_b200/build.py; this package is its Python host side (ctypes binding, layer session,
seeded synthetic inputs).
"""
__all__ = ["rvcuda", "synth"]
