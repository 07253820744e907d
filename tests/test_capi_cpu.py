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
    hdr = open(os.path.join(ROOT, "include", "rhizome_gdr.h")).read()
    declared = int(re.search(r"#define RHZ_ABI_VERSION (\d+)", hdr).group(1))
    assert lib.rhz_abi_version() == declared == 200


def test_chunk_form_setting_without_gpu(lib):
    prev = C.c_int32(-1)
    assert lib.rhz_gdr_set_chunk_kernel(7, C.byref(prev)) == capi.RHZ_ERR_INVALID
    assert b"variant 7" in lib.rhz_last_error()
    assert lib.rhz_gdr_set_chunk_kernel(capi.RHZ_CHUNK_SOLO, C.byref(prev)) == capi.RHZ_OK
    assert prev.value == capi.RHZ_CHUNK_AUTO
    assert lib.rhz_gdr_set_chunk_kernel(capi.RHZ_CHUNK_AUTO, C.byref(prev)) == capi.RHZ_OK
    assert prev.value == capi.RHZ_CHUNK_SOLO
    assert lib.rhz_gdr_set_chunk_kernel(capi.RHZ_CHUNK_GRID, C.byref(prev)) == capi.RHZ_OK
    assert lib.rhz_gdr_set_chunk_kernel(capi.RHZ_CHUNK_AUTO, C.byref(prev)) == capi.RHZ_OK
    assert prev.value == capi.RHZ_CHUNK_GRID
    assert lib.rhz_gdr_set_chunk_kernel(capi.RHZ_CHUNK_AUTO, None) == capi.RHZ_OK


def test_bwd_form_setting_without_gpu(lib):
    prev = C.c_int32(-1)
    assert lib.rhz_gdr_set_bwd_kernel(2, C.byref(prev)) == capi.RHZ_ERR_INVALID
    assert b"backward form 2" in lib.rhz_last_error()
    assert lib.rhz_gdr_set_bwd_kernel(capi.RHZ_BWD_SCAN, C.byref(prev)) == capi.RHZ_OK
    assert prev.value == capi.RHZ_BWD_AUTO
    assert lib.rhz_gdr_set_bwd_kernel(capi.RHZ_BWD_AUTO, C.byref(prev)) == capi.RHZ_OK
    assert prev.value == capi.RHZ_BWD_SCAN
    assert lib.rhz_gdr_set_bwd_kernel(capi.RHZ_BWD_AUTO, None) == capi.RHZ_OK


def test_wait_test_hook_validates_without_gpu(lib):
    assert lib.rhz_gdr_set_wait_test(2, 1000000) == capi.RHZ_ERR_INVALID
    assert lib.rhz_gdr_set_wait_test(1, 10) == capi.RHZ_ERR_INVALID  # below 1 us
    assert lib.rhz_gdr_set_wait_test(1, 3_000_000_000) == capi.RHZ_ERR_INVALID
    assert lib.rhz_gdr_set_wait_test(1, 20_000_000) == capi.RHZ_OK
    assert lib.rhz_gdr_set_wait_test(0, 0) == capi.RHZ_OK


def test_device_status_without_gpu(lib):
    assert lib.rhz_device_status(None, 0) == capi.RHZ_ERR_INVALID
    flag = C.c_int32(0)
    assert lib.rhz_device_status(C.byref(flag), 0) == capi.RHZ_ERR_DEVICE


def test_host_entry_without_gpu(lib):
    """The host-buffer scan validates on the host; T = 0 is answered there
    (the reference returns the initial state, delta.rs:135)."""
    import numpy as np
    B, H, d = 2, 3, 8
    init = np.arange(B * H * d * d, dtype=np.float32)
    fin = np.zeros_like(init)
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    st = lib.rhz_gdr_scan_chunked_host(FAKE, ptr(fin), FAKE, FAKE, FAKE, FAKE, FAKE, None,
                                       ptr(init), 64, B, 0, H, d, capi.RHZ_DTYPE_F32, None, 0,
                                       None)
    assert st == capi.RHZ_OK and np.array_equal(fin, init)
    st = lib.rhz_gdr_scan_chunked_host(FAKE, ptr(fin), FAKE, FAKE, FAKE, FAKE, FAKE, None, None,
                                       64, B, 0, H, d, capi.RHZ_DTYPE_F32, None, 0, None)
    assert st == capi.RHZ_OK and not fin.any()
    # sizes and arguments checked before any device work
    args = lambda B, T, ws, nb: (FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, 64, B, T,  # noqa: E731
                                 H, d, capi.RHZ_DTYPE_BF16, ws, nb, None)
    assert lib.rhz_gdr_scan_chunked_host(*args(70000, 4, FAKE, 1 << 40)) == capi.RHZ_ERR_SHAPE
    assert lib.rhz_gdr_scan_chunked_host(*args(2, 300, FAKE, 16)) == capi.RHZ_ERR_INVALID
    assert b"workspace too small" in lib.rhz_last_error()
    assert lib.rhz_gdr_scan_chunked_host(*args(-1, 4, FAKE, 16)) == capi.RHZ_ERR_SHAPE
    assert lib.rhz_gdr_scan_chunked_host(None, *args(2, 4, FAKE, 16)[1:]) == capi.RHZ_ERR_INVALID
    # workspace: 3 slab sets + 2 pools + whole gates + piece tables
    w = lib.rhz_gdr_host_workspace_bytes
    assert w(-1, 4, H, d, 1, 0) == 0 and w(2, 4, H, d, 9, 0) == 0
    b0, b1 = w(4, 4096, 16, 128, 1, 0), w(4, 4096, 16, 128, 1, 1)
    slab = 512
    sets = 3 * (4 * 4 * slab * 16 * 128 * 2 + 2 * 4 * slab * 16 * 4)
    assert b0 >= sets + 2 * 4 * 16 * 128 * 128 * 4 + 2 * 4 * 4096 * 16 * 4
    assert b1 > b0  # a segment change can split a slab row into more pieces
    # with a valid workspace size the call needs a device
    assert lib.rhz_gdr_scan_chunked_host(*args(2, 300, FAKE, w(2, 300, H, d, 1, 0))) == capi.RHZ_ERR_DEVICE


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
    # segment tables; plus the tensor-core kernel's rings on the bf16 d=128 path
    ws_seg = lib.rhz_gdr_workspace_bytes(4, 4096, 16, 32, capi.RHZ_DTYPE_F32, 1)
    assert ws_seg >= (4 * 4096 + 1) * 4 * 2
    assert lib.rhz_gdr_workspace_bytes(4, 4096, 16, 32, capi.RHZ_DTYPE_F32, 0) == 0
    ws_tc = lib.rhz_gdr_workspace_bytes(4, 4096, 16, 128, capi.RHZ_DTYPE_BF16, 0)
    assert ws_tc >= 128 * 8 * 32768  # 128 chains x 8 ring slots x 32 KB records
    assert lib.rhz_gdr_workspace_bytes(4, 4096, 16, 128, capi.RHZ_DTYPE_BF16, 1) > ws_tc + ws_seg // 2
    assert lib.rhz_gdr_workspace_bytes(-1, 4, 1, 4, 0, 0) == 0
    # the bf16 d=128 path refuses a missing workspace before any device work
    assert f(FAKE, None, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, 1, 64, 2, 128, 1, None, 0,
             None) == capi.RHZ_ERR_INVALID
    assert b"workspace too small" in lib.rhz_last_error()
    assert lib.rhz_gdr_scan_chunked(FAKE, None, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, -1, 1,
                                    8, 1, 4, 0, None, 0, None) == capi.RHZ_ERR_SHAPE


def test_varlen_validation(lib):
    f = lib.rhz_gdr_varlen_fwd
    base = [FAKE, FAKE, None, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 2, 10, 4, 2, 32, 0, 0, None, 0,
            None]
    bad_flags = list(base)
    bad_flags[15] = 8
    assert f(*bad_flags) == capi.RHZ_ERR_INVALID
    too_many = list(base)
    too_many[9] = 5  # 5 sequences, 4 slots, identity slot map
    assert f(*too_many) == capi.RHZ_ERR_SHAPE
    assert lib.rhz_gdr_varlen_workspace_bytes(2, 2, 32, 0) == 0
    need = lib.rhz_gdr_varlen_workspace_bytes(2, 2, 128, 1)
    assert need >= 128 * 8 * 32768 + 4 * 4  # rings + one round offset per item
    short = list(base)
    short[13], short[14], short[16], short[17] = 128, 1, FAKE, need - 256
    assert f(*short) == capi.RHZ_ERR_INVALID and b"workspace too small" in lib.rhz_last_error()
    assert lib.rhz_varlen_pack_tokens(FAKE, FAKE, FAKE, 2, 4, 6, None) == capi.RHZ_ERR_SHAPE
    assert lib.rhz_varlen_chunk_map(FAKE, FAKE, FAKE, FAKE, 2, 0, 8, FAKE, 256, None) == capi.RHZ_ERR_SHAPE


def test_python_errors_map_status_codes(lib):
    with pytest.raises(capi.ShapeError):
        capi.check(_step(lib, d=0))
    with pytest.raises(capi.DtypeError):
        capi.check(_step(lib, dtype=9))


def test_torch_wrappers_validate_before_the_library():
    """rhizome_b200.ops checks device, layout, dtype and shape of its torch
    arguments before any C-ABI call (so these run without a GPU)."""
    import torch
    from rhizome_b200 import ops
    q = torch.zeros(1, 64, 2, 128, dtype=torch.bfloat16)
    a = torch.zeros(1, 64, 2)
    with pytest.raises(capi.InvalidArgument, match="CUDA tensor"):
        ops.gdr_scan_chunked(q, q, q, a, a)
    # the host-buffer entry wants host tensors of matching shapes and dtypes
    with pytest.raises(capi.ShapeError):
        ops.gdr_scan_chunked_host(q, q[:, :32].contiguous(), q, a, a)
    with pytest.raises(capi.DtypeError):
        ops.gdr_scan_chunked_host(q, q, q, a.double(), a)
    with pytest.raises(capi.InvalidArgument, match="contiguous"):
        ops.gdr_scan_chunked_host(q.transpose(1, 2), q, q, a, a)
    with pytest.raises(capi.InvalidArgument):
        ops.set_chunk_kernel("fastest")


def test_torch_wrappers_check_out_pool_and_workspace():
    """`out=`, state pools and caller workspaces are checked against the op's
    own shapes before the library sees them (a smaller buffer would be
    written past its end on the device)."""
    import torch
    from rhizome_b200 import ops
    q = torch.zeros(4, 2, 128)
    with pytest.raises(capi.InvalidArgument, match="CUDA tensor"):
        ops._need(q, "out", q.dtype, tuple(q.shape))
    with pytest.raises(capi.ShapeError, match="expected"):
        ops._need(q[:2].contiguous(), "out", q.dtype, tuple(q.shape))
    with pytest.raises(capi.DtypeError):
        ops._need(q.bfloat16(), "out", q.dtype, tuple(q.shape))
    # state pools: trailing dims must be (H, d, d)
    pool = torch.zeros(3, 2, 64, 64)
    with pytest.raises(capi.ShapeError, match="slots"):
        ops._pool(pool, "state_pool", 2, 128)
    with pytest.raises(capi.DtypeError):
        ops._pool(torch.zeros(3, 2, 128, 128, dtype=torch.float64), "state_pool", 2, 128)
    ok = torch.zeros(3, 2, 128, 128)
    with pytest.raises(capi.InvalidArgument):
        ops._pool(ok, "state_pool", 2, 128)  # right shape, but still a host tensor
    with pytest.raises(capi.InvalidArgument, match="CUDA tensor"):
        ops._workspace(torch.zeros(16, dtype=torch.uint8), 16, torch.device("cpu"))
