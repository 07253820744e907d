"""GPU parity of the tcgen05 chunked prefill (bf16 in, fp32 state) against
the f64 oracle on the same (bf16-rounded) inputs, through the C ABI, at the
bf16 tolerance (<= 2e-2 relative to max|ref|, <= 1e-2 absolute, and
1e-2 RMS(ref) + 2e-2 |ref| elementwise). Every case runs on each form of the
kernel (the grid form: chain CTAs fed by producer CTAs through record rings;
the 2-CTA cluster per item; the one-CTA kernel), pinned through
rhz_gdr_set_chunk_kernel."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from rhizome_b200 import ops
from tests.gpu_util import chunk_form, device_inputs, host, make_inputs, to_dev
from tests.tolerance import assert_bf16

pytestmark = pytest.mark.gpu
D = 128


@pytest.fixture(autouse=True, params=["grid", "pair", "solo"])
def form(request):
    with chunk_form(request.param):
        yield request.param


def dense_case(seed, B, T, H, scale_q=1.0, alpha=None, beta=None):
    q, k, v, a, b = make_inputs(seed, B * T, H, D, "bf16")
    if scale_q != 1.0:
        q = torch.tensor(q * scale_q).to(torch.bfloat16).double().numpy()
    if alpha is not None:
        a = np.broadcast_to(np.float32(alpha), a.shape).astype(np.float64).copy()
    if beta is not None:
        b = np.broadcast_to(np.float32(beta), b.shape).astype(np.float64).copy()
    return q, k, v, a, b


def run_dense(q, k, v, a, b, B, T, **kw):
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, "bf16")
    shp = lambda x: x.reshape(B, T, *x.shape[1:])  # noqa: E731
    o, fin = ops.gdr_scan_chunked(shp(dq), shp(dk), shp(dv), shp(da), shp(db), **kw)
    torch.cuda.synchronize()
    return o, fin


@pytest.mark.parametrize("T", [1, 17, 63, 64, 65, 128, 130, 257])
def test_chunk_edges_match_oracle(T):
    B, H = 1, 2
    q, k, v, a, b = dense_case(100 + T, B, T, H)
    o, fin = run_dense(q, k, v, a, b, B, T)
    ro, rs = O.gdr_dense(*(x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b)))
    assert_bf16(host(o), ro, f"o T={T}")
    assert_bf16(host(fin), rs, f"state T={T}")


def test_reference_fixture_distribution():
    """Inputs shaped like the reference tests' make_inputs (q scaled by sqrt(d),
    alpha in [0.5, 1), beta in [0.1, 0.9)): slow decay, long memory."""
    B, T, H = 2, 300, 2
    q, k, v, a, b = make_inputs(5, B * T, H, D, "bf16")
    q = torch.tensor(q * np.sqrt(D)).to(torch.bfloat16).double().numpy()
    rng = np.random.default_rng(0)
    a = (0.5 + 0.5 * rng.random(a.shape)).astype(np.float32).astype(np.float64)
    b = (0.1 + 0.8 * rng.random(b.shape)).astype(np.float32).astype(np.float64)
    o, fin = run_dense(q, k, v, a, b, B, T)
    ro, rs = O.gdr_dense(*(x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b)))
    assert_bf16(host(o), ro, "slow-decay o", abs_bound=False)
    assert_bf16(host(fin), rs, "slow-decay state", abs_bound=False)


@pytest.mark.parametrize("alpha,beta", [(0.0, None), (1.0, 0.0), (1.0, None)])
def test_decay_edge_cases(alpha, beta):
    """alpha = 0 forgets everything each step (delta.rs:348-358); beta = 0
    writes nothing; alpha = 1 never decays."""
    B, T, H = 1, 150, 1
    q, k, v, a, b = dense_case(7, B, T, H, alpha=alpha, beta=beta)
    o, fin = run_dense(q, k, v, a, b, B, T)
    ro, rs = O.gdr_dense(*(x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b)))
    if beta == 0.0:
        assert not host(o).any() and not host(fin).any()
    assert_bf16(host(o), ro, f"o alpha={alpha}")
    assert_bf16(host(fin), rs, f"state alpha={alpha}")


def test_segments_match_reference_semantics():
    B, T, H = 2, 333, 2
    rng = np.random.default_rng(9)
    seg = np.cumsum(rng.random((B, T)) < 0.02, axis=1).astype(np.int64)
    q, k, v, a, b = dense_case(21, B, T, H)
    o, fin = run_dense(q, k, v, a, b, B, T, segment=to_dev(seg, torch.int64))
    ro = np.zeros((B, T, H, D))
    rs = np.zeros((B, H, D, D))
    qq, kk, vv, aa, bb = (x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b))
    for bi in range(B):
        for h in range(H):
            inp = O.DeltaInputs(D, qq[bi, :, h], kk[bi, :, h], vv[bi, :, h], aa[bi, :, h],
                                bb[bi, :, h], seg[bi])
            out, st = O.gated_delta_sequential(inp, O.DeltaState.zeros(D))
            ro[bi, :, h] = out.reshape(T, D)
            rs[bi, h] = st.s.reshape(D, D)
    assert_bf16(host(o), ro, "segments o")
    assert_bf16(host(fin), rs, "segments state")


def test_varlen_resumes_from_slot_states():
    """Packed continuous-batching prefill: ragged lengths (0, 1, 64, 65, ...),
    N(0, 0.02^2) initial states in a permuted slot pool, final states written
    back; the oracle is the step loop from each slot's state."""
    H, S = 4, 12
    lens = [0, 1, 64, 65, 200, 7, 1000, 129]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    q, k, v, a, b = make_inputs(31, int(cu[-1]), H, D, "bf16")
    pool = O.make_normal(4, 22, (S, H, D, D), 0.02).astype(np.float32).astype(np.float64)
    slots = np.array([11, 0, 5, 3, 8, 1, 10, 2], dtype=np.int32)
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, "bf16")
    dpool = to_dev(pool, torch.float32)
    o = ops.gdr_varlen_fwd(dq, dk, dv, da, db, to_dev(cu, torch.int32), dpool,
                           to_dev(slots, torch.int32))
    torch.cuda.synchronize()
    ro, rpool = O.gdr_varlen(cu, q, k, v, a, b, state_in=pool, state_in_index=slots,
                             state_out_index=slots)
    assert_bf16(host(o), ro, "varlen o")
    assert_bf16(host(dpool), rpool, "varlen pool")


def test_prefill_config_t512_slice_full_f64_check():
    """The chunked-prefill benchmark's shapes (B=4, H=16, d=128) on a T=512
    slice, every output and state checked against the f64 oracle."""
    B, T, H = 4, 512, 16
    q, k, v, a, b = dense_case(2025, B, T, H)
    o, fin = run_dense(q, k, v, a, b, B, T)
    ro, rs = O.gdr_dense(*(x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b)))
    assert_bf16(host(o), ro, "cfg1 T=512 o")
    assert_bf16(host(fin), rs, "cfg1 T=512 state")


def test_prefill_config_full_size():
    """B=4, T=4096, H=16, d=128 (the benchmark workload) against the f64
    oracle, plus determinism (two runs bitwise equal)."""
    B, T, H = 4, 4096, 16
    q, k, v, a, b = dense_case(2026, B, T, H)
    o, fin = run_dense(q, k, v, a, b, B, T)
    o2, fin2 = run_dense(q, k, v, a, b, B, T)
    assert torch.equal(o, o2) and torch.equal(fin, fin2), "not run-to-run deterministic"
    ro, rs = O.gdr_dense(*(x.reshape(B, T, *x.shape[1:]) for x in (q, k, v, a, b)))
    assert_bf16(host(o), ro, "cfg1 o")
    assert_bf16(host(fin), rs, "cfg1 state")


def test_batch_invariance_and_chunk_invariance():
    """A sequence's result does not depend on its batch neighbours or on the
    `chunk` argument (docs/determinism.md:3-6)."""
    B, T, H = 3, 200, 2
    q, k, v, a, b = dense_case(77, B, T, H)
    o, fin = run_dense(q, k, v, a, b, B, T, chunk=64)
    o8, fin8 = run_dense(q, k, v, a, b, B, T, chunk=8)
    assert torch.equal(o, o8) and torch.equal(fin, fin8)
    # sequence 1 alone
    sl = slice(T, 2 * T)
    o1, fin1 = run_dense(q[sl], k[sl], v[sl], a[sl], b[sl], 1, T)
    assert torch.equal(o1[0], o[1]) and torch.equal(fin1[0], fin[1])


def test_varlen_prefill_config_full_size():
    """The varlen-prefill benchmark: 64 sequences with seeded lengths
    U{1..8192} packed into one stream, H=16, d=128, bf16 inputs, each sequence
    starting from its own N(0, 0.02^2) state in a permuted slot pool and
    writing its final state back."""
    H, n = 16, 64
    rng = np.random.default_rng(8192)
    lens = rng.integers(1, 8193, size=n)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tokens = int(cu[-1])
    q, k, v, a, b = make_inputs(64, tokens, H, D, "bf16")
    S = 96
    pool = O.make_normal(6, 22, (S, H, D, D), 0.02).astype(np.float32).astype(np.float64)
    slots = rng.permutation(S)[:n].astype(np.int32)
    dq, dk, dv, da, db = device_inputs(q, k, v, a, b, "bf16")
    dpool = to_dev(pool, torch.float32)
    o = ops.gdr_varlen_fwd(dq, dk, dv, da, db, to_dev(cu, torch.int32), dpool,
                           to_dev(slots, torch.int32))
    torch.cuda.synchronize()
    ro, rpool = O.gdr_varlen(cu, q, k, v, a, b, state_in=pool, state_in_index=slots,
                             state_out_index=slots)
    assert_bf16(host(o), ro, "cfg3 o")
    assert_bf16(host(dpool), rpool, "cfg3 pool")


def test_forms_agree_and_grid_is_the_default():
    """The three forms round at the same points but accumulate the output in
    different orders (the grid form computes O^T = S Q~^T with S read from
    tensor memory), so they agree within the bf16 tolerance of each other,
    whatever the item count. "auto" is the grid form, bitwise."""
    for seed, (B, T, H) in ((55, (2, 300, 4)), (56, (2, 70, 128))):
        q, k, v, a, b = dense_case(seed, B, T, H)
        with chunk_form("pair"):
            op, sp = run_dense(q, k, v, a, b, B, T)
        with chunk_form("grid"):
            og, sg = run_dense(q, k, v, a, b, B, T)
        with chunk_form("auto"):
            oa, sa = run_dense(q, k, v, a, b, B, T)
        with chunk_form("solo"):
            os_, ss = run_dense(q, k, v, a, b, B, T)
        assert_bf16(host(og), host(op), "grid vs pair o")
        assert_bf16(host(sg), host(sp), "grid vs pair state")
        assert torch.equal(oa, og) and torch.equal(sa, sg), (B, T, H)
        assert_bf16(host(os_), host(og), "solo vs grid o")
        assert_bf16(host(ss), host(sg), "solo vs grid state")


def test_batch_invariance_of_the_default_form():
    """A sequence's output and final state do not depend on how many other
    sequences share the call (docs/determinism.md:3-6): the same sequence
    alone, among 8 items and among 256 items, bitwise."""
    T, H = 200, 2
    q, k, v, a, b = dense_case(58, 1, T, H)
    with chunk_form("auto"):
        o1, s1 = run_dense(q, k, v, a, b, 1, T)
        for B, Hx in ((4, 2), (2, 128)):
            qx, kx, vx, ax, bx = dense_case(59 + B, B, T, Hx)
            # sequence 1, heads 0..H-1 carry the probe inputs
            for dst, src in ((qx, q), (kx, k), (vx, v), (ax, a), (bx, b)):
                dst.reshape(B, T, *dst.shape[1:])[1, :, :H] = src.reshape(1, T, *src.shape[1:])[0]
            o, s = run_dense(qx, kx, vx, ax, bx, B, T)
            assert torch.equal(o[1, :, :H], o1[0]), (B, Hx)
            assert torch.equal(s[1, :H], s1[0]), (B, Hx)


def test_device_status_clear_after_runs():
    assert not ops.device_status(clear=True)
    B, T, H = 1, 130, 2
    q, k, v, a, b = dense_case(57, B, T, H)
    run_dense(q, k, v, a, b, B, T)
    assert not ops.device_status()


def test_grid_few_items_many_rounds():
    """8 items of 64 chunks: the grid form's producer contexts then take
    tasks 35 rounds apart, so a context's next ring-slot wait depends on a
    chain far ahead of the record it has just built; that record must be
    published before such a wait (a held record would stall the chain until
    the bounded waits gave up). Grid against the 2-CTA form within the bf16
    tolerance, and no device timeout."""
    from rhizome_b200 import capi
    import ctypes
    B, T, H = 2, 4096, 4
    q, k, v, a, b = dense_case(57, B, T, H)
    with chunk_form("grid"):
        og, sg = run_dense(q, k, v, a, b, B, T)
    with chunk_form("pair"):
        op, sp = run_dense(q, k, v, a, b, B, T)
    torch.cuda.synchronize()
    flag = ctypes.c_int32(-1)
    capi.call("rhz_device_status", ctypes.byref(flag), 1)
    assert flag.value == 0
    assert_bf16(host(og), host(op), "grid vs pair o")
    assert_bf16(host(sg), host(sp), "grid vs pair state")
