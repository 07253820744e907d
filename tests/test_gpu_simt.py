"""GPU parity of the SIMT kernels (ragged decode step, fp32 position-by-
position scan) against the f64 oracle, through the C ABI."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from rhizome_b200 import capi, ops
from tests.gpu_util import device_inputs, host, make_inputs, to_dev
from tests.tolerance import assert_bf16, assert_fp32

pytestmark = pytest.mark.gpu


def oracle_decode(q, k, v, a, b, states):
    """One gated_delta_step per (sequence, head) from the given states."""
    n = q.shape[0]
    cu = np.arange(n + 1)
    return O.gdr_varlen(cu, q, k, v, a, b, state_in=states)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("d", [4, 6, 32, 128, 200])
def test_decode_step_matches_oracle(dtype, d):
    n, H, slots = 37, 3, 50
    q, k, v, a, b = make_inputs(11 + d, n, H, d, dtype)
    pool = O.make_normal(5, 22, (slots, H, d, d), 0.02).astype(np.float32).astype(np.float64)
    perm = np.random.default_rng(d).permutation(slots)[:n].astype(np.int32)
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, dtype)
    dpool = to_dev(pool, torch.float32)
    dslot = to_dev(perm, torch.int32)
    o = ops.gdr_step(dq, dk, dv, da, db, dpool, dslot)
    torch.cuda.synchronize()
    ro, rs = oracle_decode(q, k, v, a, b, pool[perm])
    check = assert_fp32 if dtype == "f32" else assert_bf16
    check(host(o), ro, f"decode o d={d}")
    newpool = host(dpool)
    check(newpool[perm], rs, f"decode state d={d}")
    untouched = np.setdiff1d(np.arange(slots), perm)
    assert np.array_equal(newpool[untouched], pool[untouched])


def test_decode_full_config_shapes():
    """512 live sequences, H = 16, d = 128, a 1024-slot pool of N(0, 0.02^2)
    states and a random slot permutation (the ragged-decode benchmark)."""
    n, H, d, S = 512, 16, 128, 1024
    q, k, v, a, b = make_inputs(2024, n, H, d, "bf16")
    g = torch.Generator(device="cuda").manual_seed(7)
    dpool = torch.randn((S, H, d, d), device="cuda", generator=g) * 0.02
    perm = torch.randperm(S, device="cuda", generator=g)[:n].to(torch.int32)
    before = host(dpool[perm.long()])
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, "bf16")
    o = ops.gdr_step(dq, dk, dv, da, db, dpool, perm)
    torch.cuda.synchronize()
    ro, rs = oracle_decode(q, k, v, a, b, before)
    assert_bf16(host(o), ro, "cfg2 o")
    assert_bf16(host(dpool[perm.long()]), rs, "cfg2 state")


def test_decode_invalid_slot_writes_nan_and_keeps_pool():
    n, H, d, S = 3, 2, 32, 4
    q, k, v, a, b = make_inputs(1, n, H, d, "f32")
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, "f32")
    pool = torch.ones((S, H, d, d), device="cuda")
    slots = torch.tensor([0, 9, 2], device="cuda", dtype=torch.int32)
    o = ops.gdr_step(dq, dk, dv, da, db, pool, slots)
    torch.cuda.synchronize()
    assert torch.isnan(o[1]).all() and torch.isfinite(o[0]).all() and torch.isfinite(o[2]).all()
    assert torch.equal(pool[1], torch.ones_like(pool[1])) and torch.equal(pool[3], pool[1])


@pytest.mark.parametrize("d", [4, 6, 32, 128, 256])
def test_sequential_fp32_matches_oracle(d):
    B, T, H = 2, 150, 2
    q, k, v, a, b = make_inputs(3 + d, B * T, H, d, "f32")
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, "f32")
    shp = lambda x: x.reshape(B, T, *x.shape[1:])  # noqa: E731
    o, fin = ops.gdr_sequential(shp(dq), shp(dk), shp(dv), shp(da), shp(db))
    torch.cuda.synchronize()
    ro, rs = O.gdr_dense(*(x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b)))
    assert_fp32(host(o), ro, f"seq o d={d}")
    assert_fp32(host(fin), rs, f"seq state d={d}")


def test_sequential_fp32_long_sequence():
    B, T, H, d = 1, 4096, 4, 128
    q, k, v, a, b = make_inputs(99, B * T, H, d, "f32")
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, "f32")
    shp = lambda x: x.reshape(B, T, *x.shape[1:])  # noqa: E731
    o, fin = ops.gdr_scan_chunked(shp(dq), shp(dk), shp(dv), shp(da), shp(db), chunk=64)
    torch.cuda.synchronize()
    ro, rs = O.gdr_dense(*(x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b)))
    assert_fp32(host(o), ro, "long o")
    assert_fp32(host(fin), rs, "long state")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_sequential_with_segments_matches_reference_semantics(dtype):
    """Segment changes reset the state (delta.rs:137-141); t = 0 resets too, so
    state_init never matters; the final state is the last segment's."""
    B, T, H, d = 3, 97, 2, 32
    rng = np.random.default_rng(4)
    seg = np.cumsum(rng.random((B, T)) < 0.05, axis=1).astype(np.int64) + 7
    q, k, v, a, b = make_inputs(8, B * T, H, d, dtype)
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, dtype)
    shp = lambda x: x.reshape(B, T, *x.shape[1:])  # noqa: E731
    init = torch.full((B, H, d, d), 3.0, device="cuda")
    o, fin = ops.gdr_sequential(shp(dq), shp(dk), shp(dv), shp(da), shp(db),
                                segment=to_dev(seg, torch.int64), state_init=init)
    torch.cuda.synchronize()
    ro = np.zeros((B, T, H, d))
    rs = np.zeros((B, H, d, d))
    qq, kk, vv, aa, bb = (x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b))
    for bi in range(B):
        for h in range(H):
            inp = O.DeltaInputs(d, qq[bi, :, h], kk[bi, :, h], vv[bi, :, h], aa[bi, :, h],
                                bb[bi, :, h], seg[bi])
            out, st = O.gated_delta_sequential(inp, O.DeltaState(d, np.full(d * d, 3.0)))
            ro[bi, :, h] = out.reshape(T, d)
            rs[bi, h] = st.s.reshape(d, d)
    check = assert_fp32 if dtype == "f32" else assert_bf16
    check(host(o), ro, "segments o")
    check(host(fin), rs, "segments state")


def test_sequential_empty_T_returns_init_like_reference():
    B, H, d = 2, 2, 8
    q = torch.zeros((B, 0, H, d), device="cuda")
    al = torch.zeros((B, 0, H), device="cuda")
    init = torch.randn((B, H, d, d), device="cuda")
    o, fin = ops.gdr_sequential(q, q, q, al, al, state_init=init)
    torch.cuda.synchronize()
    assert o.numel() == 0 and torch.equal(fin, init)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_varlen_fwd_resumes_from_slots(dtype):
    d, H, S = 64, 2, 9
    lens = [0, 1, 63, 64, 130, 7]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tokens = int(cu[-1])
    q, k, v, a, b = make_inputs(17, tokens, H, d, dtype)
    pool = O.make_normal(3, 22, (S, H, d, d), 0.02).astype(np.float32).astype(np.float64)
    slots = np.array([4, 0, 8, 2, 6, 1], dtype=np.int32)
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, dtype)
    dpool = to_dev(pool, torch.float32)
    o = ops.gdr_varlen_fwd(dq, dk, dv, da, db, to_dev(cu, torch.int32), dpool,
                           to_dev(slots, torch.int32))
    torch.cuda.synchronize()
    ro, rpool = O.gdr_varlen(cu, q, k, v, a, b, state_in=pool, state_in_index=slots,
                             state_out_index=slots)
    check = assert_fp32 if dtype == "f32" else assert_bf16
    check(host(o), ro, "varlen o")
    check(host(dpool), rpool, "varlen pool")


def test_varlen_zero_init_and_no_write():
    d, H, S = 32, 1, 3
    cu = np.array([0, 5, 12], dtype=np.int32)
    q, k, v, a, b = make_inputs(2, 12, H, d, "f32")
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, "f32")
    dpool = torch.full((S, H, d, d), 2.0, device="cuda")
    o = ops.gdr_varlen_fwd(dq, dk, dv, da, db, to_dev(cu, torch.int32), dpool, None,
                           zero_init=True, write_state=False)
    torch.cuda.synchronize()
    ro, _ = O.gdr_varlen(cu, q, k, v, a, b)
    assert_fp32(host(o), ro, "zero-init o")
    assert torch.equal(dpool, torch.full_like(dpool, 2.0))


def test_shape_errors_raise_before_launch():
    q = torch.zeros((2, 3, 1, 8), device="cuda")
    al = torch.zeros((2, 3, 1), device="cuda")
    with pytest.raises(capi.ShapeError):
        ops.gdr_sequential(q, q, q, al, torch.zeros((2, 4, 1), device="cuda"))
    with pytest.raises(capi.DtypeError):
        ops.gdr_sequential(q.half(), q.half(), q.half(), al, al)


def test_wrappers_check_out_pools_and_workspaces():
    """A too-small `out`, a state pool of the wrong head count or width, or a
    too-small caller workspace is rejected before the library writes past its
    end."""
    n, H, d = 4, 2, 32
    q = torch.zeros((n, H, d), device="cuda")
    g = torch.zeros((n, H), device="cuda")
    pool = torch.zeros((n, H, d, d), device="cuda")
    with pytest.raises(capi.ShapeError):
        ops.gdr_step(q, q, q, g, g, pool, out=q[:2].clone())
    with pytest.raises(capi.DtypeError):
        ops.gdr_step(q, q, q, g, g, pool, out=q.bfloat16())
    cu = torch.tensor([0, 2, 4], device="cuda", dtype=torch.int32)
    with pytest.raises(capi.ShapeError, match="slots"):
        ops.gdr_varlen_fwd(q, q, q, g, g, cu, state_pool=torch.zeros((n, 1, d, d), device="cuda"))
    with pytest.raises(capi.ShapeError):
        ops.gdr_varlen_fwd(q, q, q, g, g, cu, state_pool=pool, out=q[:, :1].clone())
    x = torch.zeros((2, 8, H, d), device="cuda")
    a = torch.zeros((2, 8, H), device="cuda")
    seg = torch.zeros((2, 8), device="cuda", dtype=torch.int64)
    small = torch.empty(8, device="cuda", dtype=torch.uint8)
    with pytest.raises(capi.InvalidArgument, match="workspace"):
        ops.gdr_sequential(x, x, x, a, a, segment=seg, workspace=small)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("d", [6, 32, 128])
def test_multistep_reference_semantics(dtype, d):
    """gated_delta_multistep (delta.rs:201-230): zero start, resets at segment
    changes, every per-position state returned."""
    n, T, H, maxp = 5, 10, 2, 8
    q, k, v, a, b = make_inputs(40 + d, n * T, H, d, dtype)
    rng = np.random.default_rng(d)
    seg = np.cumsum(rng.random((n, T)) < 0.25, axis=1).astype(np.int64)
    sh = lambda x: x.reshape(n, T, *x.shape[1:])  # noqa: E731
    dq, dk, dv, da, db = (sh(x) for x in device_inputs(q, k, v, a, b, dtype))
    outs, states = ops.gdr_multistep(dq, dk, dv, da, db, max_positions=maxp,
                                     segment=to_dev(seg, torch.int64))
    torch.cuda.synchronize()
    check = assert_fp32 if dtype == "f32" else assert_bf16
    qq, kk, vv, aa, bb = (sh(x) for x in (q, k, v, a, b))
    for i in range(n):
        for h in range(H):
            inp = O.DeltaInputs(d, qq[i, :, h], kk[i, :, h], vv[i, :, h], aa[i, :, h],
                                bb[i, :, h], seg[i])
            ro, rst = O.gated_delta_multistep(inp, O.DeltaState.zeros(d), maxp)
            check(host(outs[i, :, h]).ravel(), ro, f"multistep o {i} {h}")
            for t, st in enumerate(rst):
                check(host(states[i, t, h]).ravel(), st.s, f"multistep state {i} {h} {t}")


def test_multistep_from_slots_leaves_pool_untouched():
    n, T, H, d, S = 4, 6, 3, 128, 7
    q, k, v, a, b = make_inputs(77, n * T, H, d, "bf16")
    pool = O.make_normal(9, 22, (S, H, d, d), 0.02).astype(np.float32).astype(np.float64)
    slots = np.array([6, 1, 4, 2], dtype=np.int32)
    sh = lambda x: x.reshape(n, T, *x.shape[1:])  # noqa: E731
    dq, dk, dv, da, db = (sh(x) for x in device_inputs(q, k, v, a, b, "bf16"))
    dpool = to_dev(pool, torch.float32)
    before = dpool.clone()
    outs, states = ops.gdr_multistep(dq, dk, dv, da, db, max_positions=8, state_pool=dpool,
                                     slot_idx=to_dev(slots, torch.int32))
    torch.cuda.synchronize()
    assert torch.equal(dpool, before)
    cu = np.arange(0, n * T + 1, T)
    ro, _ = O.gdr_varlen(cu, q, k, v, a, b, state_in=pool, state_in_index=slots)
    assert_bf16(host(outs).reshape(n * T, H, d), ro, "multistep from slots")
    # the last per-position state is the step loop's final state
    _, rfin = O.gdr_varlen(cu, q, k, v, a, b, state_in=pool, state_in_index=slots,
                           state_out_shape=(n, H, d, d))
    assert_bf16(host(states[:, -1]), rfin, "multistep final state")
