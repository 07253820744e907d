"""The C-ABI library on a host without a GPU: it loads, exports every symbol
include/rhizome_gdr.h declares, and rejects bad arguments with the right
status before touching a device."""
import ctypes as C
import os
import re
import subprocess

import pytest

from rhizome_b200 import build, capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for hdr in os.listdir(os.path.join(ROOT, "include")):
        if hdr.endswith(".h"):
            src = open(os.path.join(ROOT, "include", hdr)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(rhz_\w+)\s*\(", src))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    build.build()
    return capi.lib()


def test_library_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert len(syms) >= 14
    out = subprocess.run(["nm", "-D", "--defined-only", capi.lib_path()], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (rhz_\w+)", out))
    missing = [s for s in syms if s not in exported]
    assert not missing, missing
    for s in syms:
        assert getattr(lib, s) is not None
    assert set(capi.SIGNATURES) == set(syms), "capi.SIGNATURES out of sync with the header"


def test_library_does_not_depend_on_torch_or_libcuda():
    out = subprocess.run(["ldd", capi.lib_path()], capture_output=True, text=True).stdout
    assert "torch" not in out and "libcuda.so" not in out


def test_abi_version(lib):
    assert lib.rhz_abi_version() == 100


FAKE = 1 << 20  # an aligned non-null address; never dereferenced by validation


def _step(lib, **kw):
    a = dict(o=FAKE, pool=FAKE, slots=None, q=FAKE, k=FAKE, v=FAKE, al=FAKE, be=FAKE, n=4,
             num_slots=8, H=2, d=32, dtype=capi.RHZ_DTYPE_F32)
    a.update(kw)
    return lib.rhz_gdr_step(a["o"], a["pool"], a["slots"], a["q"], a["k"], a["v"], a["al"],
                            a["be"], a["n"], a["num_slots"], a["H"], a["d"], a["dtype"], None)


def test_step_rejects_bad_shapes_without_gpu(lib):
    assert _step(lib, d=0) == capi.RHZ_ERR_SHAPE  # head_dim > 0 (delta.rs:50)
    assert _step(lib, d=257) == capi.RHZ_ERR_SHAPE
    assert _step(lib, H=0) == capi.RHZ_ERR_SHAPE
    assert _step(lib, n=-1) == capi.RHZ_ERR_SHAPE
    assert _step(lib, n=9, num_slots=8) == capi.RHZ_ERR_SHAPE
    assert b"slots" in lib.rhz_last_error()
    assert _step(lib, dtype=7) == capi.RHZ_ERR_DTYPE
    assert _step(lib, q=None) == capi.RHZ_ERR_INVALID
    assert _step(lib, k=FAKE + 2) == capi.RHZ_ERR_INVALID
    assert _step(lib, n=0) == capi.RHZ_OK  # empty batch: nothing to do
    assert lib.rhz_last_error() == b""


def test_valid_call_without_gpu_reports_device_error(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _step(lib) == capi.RHZ_ERR_DEVICE
    assert lib.rhz_last_error() != b""


def test_sequential_validation(lib):
    f = lib.rhz_gdr_sequential
    args = lambda **kw: dict(dict(o=FAKE, fin=None, q=FAKE, k=FAKE, v=FAKE, al=FAKE, be=FAKE,  # noqa
                                  seg=None, init=None, B=1, T=8, H=1, d=4, dt=0, ws=None, wsb=0), **kw)

    def call(**kw):
        a = args(**kw)
        return f(a["o"], a["fin"], a["q"], a["k"], a["v"], a["al"], a["be"], a["seg"], a["init"],
                 a["B"], a["T"], a["H"], a["d"], a["dt"], a["ws"], a["wsb"], None)

    assert call(T=-1) == capi.RHZ_ERR_SHAPE
    assert call(d=0) == capi.RHZ_ERR_SHAPE
    assert call(dt=2) == capi.RHZ_ERR_DTYPE
    assert call(seg=FAKE + 4) == capi.RHZ_ERR_INVALID  # int64 ids need 8-byte alignment
    assert call(B=0) == capi.RHZ_OK or call(B=0) == capi.RHZ_ERR_DEVICE
    ws = lib.rhz_gdr_workspace_bytes(4, 4096)
    assert ws >= (4 * 4096 + 1) * 4 * 2
    assert lib.rhz_gdr_scan_chunked(FAKE, None, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, -1, 1,
                                    8, 1, 4, 0, None, 0, None) == capi.RHZ_ERR_SHAPE


def test_varlen_validation(lib):
    f = lib.rhz_gdr_varlen_fwd
    base = [FAKE, FAKE, None, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 2, 10, 4, 2, 32, 0, 0, None]
    bad_flags = list(base)
    bad_flags[15] = 8
    assert f(*bad_flags) == capi.RHZ_ERR_INVALID
    too_many = list(base)
    too_many[9] = 5  # 5 sequences, 4 slots, identity slot map
    assert f(*too_many) == capi.RHZ_ERR_SHAPE
    assert lib.rhz_varlen_pack_tokens(FAKE, FAKE, FAKE, 2, 4, 6, None) == capi.RHZ_ERR_SHAPE
    assert lib.rhz_varlen_chunk_map(FAKE, FAKE, FAKE, FAKE, 2, 0, 8, FAKE, 256, None) == capi.RHZ_ERR_SHAPE


def test_python_errors_map_status_codes(lib):
    with pytest.raises(capi.ShapeError):
        capi.check(_step(lib, d=0))
    with pytest.raises(capi.DtypeError):
        capi.check(_step(lib, dtype=9))
