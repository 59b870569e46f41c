"""clusterlm_b200 — B200-native speculative-window backend for ClusterLM.

The compute lives in libclm_b200.so (hand-written sm_100a CUDA behind the C ABI in include/clm_b200.h).
This package is a thin Python face of that ABI; importing it fails if the library is not built.
"""
from ._native import ClmError, LIB_PATH, exported_symbols  # noqa: F401

__all__ = ["ClmError", "LIB_PATH", "exported_symbols"]
