"""g4w4: B200-native (sm_100a) W4A16 hot path of gemma4-js behind a C ABI.

Import as `importlib.import_module("gemma4-js_b200")`.  `runtime` mirrors the
reference's GPU operator API (GPUOps.w4 / attention, GPUW4Linear, pleRowsToGpu,
KVCache) over libg4w4.so; `build` compiles the library in-tree.
"""
from ._lib import G4Error, load  # noqa: F401

__all__ = ["G4Error", "load"]
