"""B200 (sm_100a) backend for RHIZOME's gated delta-rule (GDR) op.

The compute lives in librhizome_gdr.so (CUDA C++ behind the C ABI in
include/rhizome_gdr.h); this package binds it (capi), wraps it for torch
device tensors (ops) and mirrors the reference's Rust API (delta).
"""
from . import capi  # noqa: F401

__all__ = ["capi", "ops", "delta", "build"]
