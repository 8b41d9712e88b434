"""wginfer_b200 — a B200 (sm_100a) device backend for the wGInfer decode path.

``wginfer_b200.ops`` mirrors the reference's op surface over torch CUDA
tensors; ``wginfer_b200.qwen2`` is the Qwen2 decoder that calls it. Both go
through the C-ABI in include/wginfer_b200.h (libwginfer_b200.so).
"""
from ._lib import NUMERICS_FAST, NUMERICS_REFERENCE, WgbError, get_numerics, numerics, set_numerics  # noqa: F401

__all__ = ["ops", "numerics", "set_numerics", "get_numerics", "NUMERICS_FAST", "NUMERICS_REFERENCE", "WgbError"]
