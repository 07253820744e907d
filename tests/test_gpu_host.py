"""GPU parity of the host-buffer entry point (rhz_gdr_scan_chunked_host):
host tensors in, host tensors out, the copies pipelined over slabs of
positions. Without segments its results are bitwise those of the device
entry point (slabs start on chunk boundaries, the fp32 state crosses them
unrounded); with segments they match the f64 oracle at the path's
tolerance."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from rhizome_b200 import ops
from tests.gpu_util import make_inputs
from tests.tolerance import assert_bf16, assert_fp32

pytestmark = pytest.mark.gpu
TD = {"bf16": torch.bfloat16, "f32": torch.float32}


def host_inputs(seed, B, T, H, d, dtype, pin=True):
    q, k, v, a, b = make_inputs(seed, B * T, H, d, dtype)
    shp = lambda x: x.reshape(B, T, *x.shape[1:])  # noqa: E731
    cpu = [torch.from_numpy(np.ascontiguousarray(shp(x))).to(TD[dtype]) for x in (q, k, v)]
    cpu += [torch.from_numpy(np.ascontiguousarray(shp(x))).float() for x in (a, b)]
    if pin:
        cpu = [x.pin_memory() for x in cpu]
    return [shp(x) for x in (q, k, v, a, b)], cpu


def oracle_segmented(q, k, v, a, b, seg):
    B, T, H, d = q.shape
    ro = np.zeros((B, T, H, d))
    rs = np.zeros((B, H, d, d))
    for bi in range(B):
        for h in range(H):
            inp = O.DeltaInputs(d, q[bi, :, h], k[bi, :, h], v[bi, :, h], a[bi, :, h], b[bi, :, h],
                                None if seg is None else seg[bi])
            out, st = O.gated_delta_sequential(inp, O.DeltaState.zeros(d))
            ro[bi, :, h] = out.reshape(T, d)
            rs[bi, h] = st.s.reshape(d, d)
    return ro, rs


@pytest.mark.parametrize("dtype,d", [("bf16", 128), ("f32", 64)])
@pytest.mark.parametrize("T", [1, 255, 1000])
def test_bitwise_equal_to_device_entry(dtype, d, T):
    B, H = 2, 3
    ref_np, cpu = host_inputs(T + d, B, T, H, d, dtype)
    o, fin = ops.gdr_scan_chunked_host(*cpu)
    dev = [x.cuda() for x in cpu]
    do, dfin = ops.gdr_scan_chunked(*dev)
    torch.cuda.synchronize()
    assert torch.equal(o, do.cpu()) and torch.equal(fin, dfin.cpu())
    ro, rs = O.gdr_dense(*ref_np)
    chk = assert_bf16 if dtype == "bf16" else assert_fp32
    chk(o.double().numpy(), ro, f"host o T={T}")
    chk(fin.double().numpy(), rs, f"host state T={T}")


@pytest.mark.parametrize("dtype,d", [("bf16", 128), ("f32", 32)])
def test_segments_across_slab_boundaries(dtype, d):
    """Segment changes inside slabs, exactly on a slab start (t = 256) and
    segments that run across slab boundaries (carried state)."""
    B, T, H = 3, 777, 2
    ref_np, cpu = host_inputs(17, B, T, H, d, dtype)
    rng = np.random.default_rng(3)
    seg = np.cumsum(rng.random((B, T)) < 0.01, axis=1).astype(np.int64)
    seg[0, 256:] += 100   # a change exactly on the second slab's start
    seg[1, :] = 7         # one segment through every slab
    cseg = torch.from_numpy(seg)
    o, fin = ops.gdr_scan_chunked_host(*cpu, segment=cseg)
    ro, rs = oracle_segmented(*ref_np, seg)
    if dtype == "bf16":
        assert_bf16(o.double().numpy(), ro, "host segments o")
        assert_bf16(fin.double().numpy(), rs, "host segments state")
    else:
        # the fp32 kernel is position-serial: slabs change nothing
        do, dfin = ops.gdr_scan_chunked(*(x.cuda() for x in cpu), segment=cseg.cuda())
        assert torch.equal(o, do.cpu()) and torch.equal(fin, dfin.cpu())
        assert_fp32(o.double().numpy(), ro, "host segments o")
        assert_fp32(fin.double().numpy(), rs, "host segments state")


def test_pageable_host_memory_and_edge_sizes():
    B, T, H, d = 2, 300, 2, 128
    _, cpu = host_inputs(5, B, T, H, d, "bf16", pin=False)
    o, fin = ops.gdr_scan_chunked_host(*cpu)
    do, dfin = ops.gdr_scan_chunked(*(x.cuda() for x in cpu))
    assert torch.equal(o, do.cpu()) and torch.equal(fin, dfin.cpu())
    # T = 0: the reference returns the initial state (delta.rs:135)
    z = [x[:, :0].contiguous() for x in cpu]
    init = torch.randn(B, H, d, d)
    o0, f0 = ops.gdr_scan_chunked_host(*z, state_init=init)
    assert o0.numel() == 0 and torch.equal(f0, init)
    # B = 0
    e = [x[:0].contiguous() for x in cpu]
    o1, f1 = ops.gdr_scan_chunked_host(*e)
    assert o1.numel() == 0 and f1.numel() == 0


def test_benchmark_shape_bitwise():
    """B=4, T=4096, H=16, d=128 (eight 512-position slabs) against the device
    entry point, bitwise."""
    B, T, H, d = 4, 4096, 16, 128
    g = torch.Generator().manual_seed(11)
    n = torch.nn.functional.normalize
    q = n(torch.randn(B, T, H, d, generator=g), dim=-1).bfloat16().pin_memory()
    k = n(torch.randn(B, T, H, d, generator=g), dim=-1).bfloat16().pin_memory()
    v = torch.randn(B, T, H, d, generator=g).bfloat16().pin_memory()
    b = torch.sigmoid(torch.randn(B, T, H, generator=g)).pin_memory()
    a = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, generator=g) + 2)).pin_memory()
    o, fin = ops.gdr_scan_chunked_host(q, k, v, a, b)
    do, dfin = ops.gdr_scan_chunked(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda())
    assert torch.equal(o, do.cpu()) and torch.equal(fin, dfin.cpu())


def test_rejects_device_tensors_and_small_workspace():
    _, cpu = host_inputs(6, 1, 64, 1, 128, "bf16")
    with pytest.raises(Exception):
        ops.gdr_scan_chunked_host(cpu[0].cuda(), *cpu[1:])
    ws = torch.empty(16, device="cuda", dtype=torch.uint8)
    with pytest.raises(Exception, match="workspace too small"):
        ops.gdr_scan_chunked_host(*cpu, workspace=ws)
