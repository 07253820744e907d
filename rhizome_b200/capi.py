"""ctypes binding of include/rhizome_gdr.h (the library's C ABI).

Loads rhizome_b200/_lib/librhizome_gdr.so. There is no fallback: if the
library is missing the import of any op raises, naming the build command.
Status codes become exceptions carrying the library's message.
"""
from __future__ import annotations

import ctypes as C
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "librhizome_gdr.so")

RHZ_OK = 0
RHZ_ERR_SHAPE = 1
RHZ_ERR_INVALID = 2
RHZ_ERR_DTYPE = 3
RHZ_ERR_DEVICE = 4
RHZ_ERR_TIMEOUT = 5
RHZ_ERR_NCCL = 6

RHZ_DTYPE_F32 = 0
RHZ_DTYPE_BF16 = 1

RHZ_FLAG_ZERO_INIT = 1
RHZ_FLAG_NO_STATE_WRITE = 2


class RhzError(RuntimeError):
    """A non-OK status from the library."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class ShapeError(RhzError, ValueError):
    """Shape mismatch: the counterpart of rhizome_core::Error::Shape."""


class InvalidArgument(RhzError, ValueError):
    pass


class DtypeError(RhzError, TypeError):
    pass


class DeviceError(RhzError):
    pass


class DeviceTimeout(RhzError):
    pass


_ERRORS = {RHZ_ERR_SHAPE: ShapeError, RHZ_ERR_INVALID: InvalidArgument,
           RHZ_ERR_DTYPE: DtypeError, RHZ_ERR_DEVICE: DeviceError,
           RHZ_ERR_TIMEOUT: DeviceTimeout}

# Every symbol the header declares, with (restype, argtypes).
_vp, _i32, _i64, _u32, _sz = C.c_void_p, C.c_int32, C.c_int64, C.c_uint32, C.c_size_t
SIGNATURES = {
    "rhz_last_error": (C.c_char_p, []),
    "rhz_abi_version": (C.c_int, []),
    "rhz_gdr_step": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32,
                               _i32, _vp]),
    "rhz_gdr_sequential": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                     _i32, _i32, _i32, _vp, _sz, _vp]),
    "rhz_gdr_scan_chunked": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                       _i64, _i32, _i32, _i32, _vp, _sz, _vp]),
    "rhz_gdr_varlen_fwd": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                     _i64, _i32, _i32, _i32, _u32, _vp, _sz, _vp]),
    "rhz_gdr_varlen_workspace_bytes": (_sz, [_i64, _i32, _i32, _i32]),
    "rhz_gdr_workspace_bytes": (_sz, [_i64, _i64, _i32, _i32, _i32, C.c_int]),
    "rhz_gdr_multistep": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                    _i64, _i64, _i32, _i32, _i32, _vp]),
    "rhz_varlen_prefix_sum": (C.c_int, [_vp, _vp, _i64, _vp]),
    "rhz_varlen_segments_to_cu_seqlens": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _vp, _sz, _vp]),
    "rhz_varlen_chunk_map": (C.c_int, [_vp, _vp, _vp, _vp, _i64, _i32, _i64, _vp, _sz, _vp]),
    "rhz_varlen_workspace_bytes": (_sz, [_i64]),
    "rhz_varlen_gather_states": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _vp]),
    "rhz_varlen_scatter_states": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _vp]),
    "rhz_varlen_pack_tokens": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "rhz_varlen_unpack_tokens": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "rhz_varlen_segments_to_cu_seqlens_noalloc": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "rhz_gdr_varlen_fwd_norm": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                          C.c_float, _i64, _i64, _i64, _i32, _i32, _i32,
                                          C.c_uint32, _vp, _sz, _vp]),
    "rhz_gdr_scan_chunked_bwd": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                           _vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _vp, _sz,
                                           _vp]),
    "rhz_gdr_bwd_workspace_bytes": (_sz, [_i64, _i64, _i32, _i32]),
    "rhz_groupnorm_heads": (C.c_int, [_vp, _vp, _vp, _i64, _i32, _i32, C.c_float, _i32, _vp]),
    "rhz_gdr_prep": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                               _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, C.c_float, _i32,
                               C.c_uint32, _vp]),
    "rhz_heads_unshard": (C.c_int, [_vp, _vp, _i64, _i64, _i32, _i32, _i32, _vp]),
    "rhz_heads_shard": (C.c_int, [_vp, _vp, _i64, _i64, _i32, _i32, _i32, _vp]),
    "rhz_device_status": (C.c_int, [_vp, C.c_int]),
    "rhz_gdr_scan_chunked_host": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64,
                                            _i64, _i64, _i32, _i32, _i32, _vp, _sz, _vp]),
    "rhz_gdr_host_workspace_bytes": (_sz, [_i64, _i64, _i32, _i32, _i32, C.c_int]),
    "rhz_gdr_set_chunk_kernel": (C.c_int, [_i32, _vp]),
    "rhz_gdr_set_bwd_kernel": (C.c_int, [_i32, _vp]),
    "rhz_gdr_set_wait_test": (C.c_int, [_i32, _i64]),
}

# Forms of the tensor-core chunked scan (enum rhz_chunk_kernel).
RHZ_CHUNK_AUTO, RHZ_CHUNK_PAIR, RHZ_CHUNK_SOLO, RHZ_CHUNK_GRID = 0, 1, 2, 3
RHZ_BWD_AUTO, RHZ_BWD_SCAN = 0, 1

# Largest B*T rhz_varlen_segments_to_cu_seqlens_noalloc accepts.
RHZ_NOALLOC_MAX_POSITIONS = 1 << 26

_lib = None


def lib_path() -> str:
    return _LIB_PATH


def lib():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise ImportError(f"{_LIB_PATH} is missing: run `python -m rhizome_b200.build` "
                              "(the GDR ops have no fallback path)")
        L = C.CDLL(_LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != RHZ_OK:
        msg = lib().rhz_last_error().decode(errors="replace")
        raise _ERRORS.get(status, RhzError)(status, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
