"""unpopped_b200 — the sm_100a (B200) execution backend for Unpopped's lifted kernel families.

The product is libunpopped_sm100.so (C ABI: include/up_sm100.h), hand-written CUDA for sm_100a. This package
binds it: `backend.CudaSm100` answers the reference's Backend seam, `ops` runs each kernel family on torch
CUDA tensors, and `dist` shards the families over the GPUs of one node (one process per GPU).
"""
from . import _lib  # noqa: F401

__all__ = ["backend", "ops", "dist", "build"]
