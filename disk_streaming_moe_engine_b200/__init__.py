"""B200-native (sm_100a) decode step of DISMOEN behind the C ABI libdismoen_cuda.so.

The compute path is the in-tree CUDA library; importing the package does not load it,
`Engine(...)` does, and fails loudly when the library is missing (no CPU fallback).
"""
from .config import ModelConfig, RuntimeConfig, preset  # noqa: F401
from .engine import Engine, GatedAttnKVCache, GDNState, RoutingInfo  # noqa: F401
from ._lib import DmError, load as load_library  # noqa: F401

__all__ = ["ModelConfig", "RuntimeConfig", "preset", "Engine", "GatedAttnKVCache", "GDNState",
           "RoutingInfo", "DmError", "load_library"]
