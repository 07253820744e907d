"""Pins the f64 oracle (oracle/gdr_oracle.c) to the reference.

Every test the reference holds for this path is restated here against the
oracle (crates/ops/src/delta.rs:245-369, crates/ops/src/rng.rs:109-182), then
closed-form cases and a bit-exact cross-check against a pure-Python
transcription of the same Rust code.
"""
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests import ref_python

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def segs_zero(t):
    return [0] * t


# ---------------------------------------------------------------- delta.rs tests

def test_inputs_validate_shapes():  # delta.rs:282-287
    inp = O.make_inputs(4, 3, [0, 0, 0, 0], 1)
    assert inp.is_consistent()
    assert not inp.is_empty()
    bad = O.DeltaInputs(3, inp.q[:-1], inp.k, inp.v, inp.alpha, inp.beta, inp.segment)
    assert not bad.is_consistent()
    assert not O.DeltaInputs(0, [], [], [], [], [], []).is_consistent()


def test_chunked_matches_sequential_single_segment():  # delta.rs:289-303
    t, d = 40, 6
    inp = O.make_inputs(t, d, segs_zero(t), 2)
    init = O.DeltaState.zeros(d)
    a, sa = O.gated_delta_sequential(inp, init)
    for chunk in [1, 3, 8, 64]:
        b, sb = O.gated_delta_scan_chunked(inp, init, chunk)
        assert np.all(np.abs(a - b) < 1e-10), chunk
        assert sa.max_abs_diff(sb) < 1e-10


def test_chunked_matches_sequential_with_segments():  # delta.rs:305-317
    d = 4
    segs = [0, 0, 0, 1, 1, 2, 2, 2, 2, 3]
    inp = O.make_inputs(len(segs), d, segs, 3)
    init = O.DeltaState.zeros(d)
    a, sa = O.gated_delta_sequential(inp, init)
    b, sb = O.gated_delta_scan_chunked(inp, init, 4)
    assert np.all(np.abs(a - b) < 1e-10)
    assert sa.max_abs_diff(sb) < 1e-10


def test_multistep_matches_repeated_step():  # delta.rs:319-331
    d, t = 5, 8
    inp = O.make_inputs(t, d, segs_zero(t), 4)
    init = O.DeltaState.zeros(d)
    outs, states = O.gated_delta_multistep(inp, init, 8)
    seq, final_state = O.gated_delta_sequential(inp, init)
    assert np.all(np.abs(outs - seq) < 1e-12)
    assert states[t - 1].max_abs_diff(final_state) < 1e-12


def test_segment_reset_makes_history_irrelevant():  # delta.rs:333-346
    d = 3
    segs = [0, 0, 1, 1]
    inp = O.make_inputs(4, d, segs, 5)
    dirty = O.DeltaState.zeros(d)
    dirty.s[:] = 3.0
    a, _ = O.gated_delta_sequential(inp, O.DeltaState.zeros(d))
    b, _ = O.gated_delta_sequential(inp, dirty)
    for i in range(2 * d, 4 * d):
        assert abs(a[i] - b[i]) < 1e-12


def test_alpha_zero_forgets_the_past():  # delta.rs:348-358
    d = 3
    s = O.DeltaState.zeros(d)
    s.s[:] = 1.0
    o = O.gated_delta_step(s, [1.0, 1.0, 1.0], [1.0, 0.0, 0.0], [0.0, 0.0, 0.0], 0.0, 0.5)
    assert np.all(np.abs(o) < 1e-12)


def test_conv_state_shifts():  # delta.rs:360-369
    st = np.zeros(3)
    w = [0.1, 0.2, 0.3, 0.4]
    y0 = O.causal_conv1d_step(st, w, 1.0, 0.0)
    assert abs(y0 - 0.4) < 1e-12
    y1 = O.causal_conv1d_step(st, w, 1.0, 0.0)
    assert abs(y1 - 0.7) < 1e-12
    assert list(st) == [0.0, 1.0, 1.0]


# ---------------------------------------------------------------- rng.rs tests

def test_philox_is_reproducible():  # rng.rs:113-124
    assert np.array_equal(O.Philox(7, 1).u32(16), O.Philox(7, 1).u32(16))


def test_philox_streams_are_independent():  # rng.rs:126-133
    assert not np.array_equal(O.Philox(7, 1).u32(8), O.Philox(7, 2).u32(8))


def test_philox_seek_gives_position_independence():  # rng.rs:135-145
    words = O.Philox(11, 3).u32(41)
    expected = words[40]
    # seek(10) then next_u32 == word 40 (block 10, lane 0)
    b = O.philox_block(0, 11, 10, 3)
    assert b[0] == expected


def test_philox_uniform_is_in_range():  # rng.rs:147-154
    u = O.Philox(1, 1).f64(10_000)
    assert np.all((u >= 0.0) & (u < 1.0))


def test_philox_normal_has_expected_moments():  # rng.rs:156-165
    xs = O.Philox(5, 9).normal(20_000)
    mean = xs.mean()
    var = ((xs - mean) ** 2).mean()
    assert abs(mean) < 0.05
    assert abs(var - 1.0) < 0.1


def test_stateless_matches_stateful_block():  # rng.rs:176-181
    v = O.stateless_uniform(2, 3, 4)
    assert 0.0 <= v < 1.0
    assert abs(O.stateless_uniform(2, 3, 4) - v) < 1e-18
    b = O.philox_block(0, 2, 4, 3)
    assert v == ((int(b[0]) >> 5 << 26) | (int(b[1]) >> 6)) / float(1 << 53)


def test_philox_block_matches_curand_fixture():
    """Cross-implementation pin: cuRAND's Philox4x32-10 block function, run on
    a B200 by tests/golden/make_philox_kat.py, gives the same words."""
    path = os.path.join(GOLDEN, "philox_kat.json")
    if not os.path.exists(path):
        pytest.skip("philox_kat.json not generated yet")
    with open(path) as f:
        kat = json.load(f)
    assert kat["cases"], "empty fixture"
    for case in kat["cases"]:
        got = O.philox_block(case["key"][0], case["key"][1],
                             case["ctr"][0] | (case["ctr"][1] << 32),
                             case["ctr"][2] | (case["ctr"][3] << 32))
        assert [int(x) for x in got] == case["out"], case


# ---------------------------------------------------------------- closed forms

def test_scalar_head_closed_form():
    """d = 1: S_t = alpha (S - beta S k k) + beta v k, o = S q."""
    rng = np.random.default_rng(0)
    t = 50
    q, k, v = rng.normal(size=t), rng.normal(size=t), rng.normal(size=t)
    al, be = rng.uniform(0.2, 1, size=t), rng.uniform(0.1, 0.9, size=t)
    inp = O.DeltaInputs(1, q, k, v, al, be, np.zeros(t, np.int64))
    out, fin = O.gated_delta_sequential(inp, O.DeltaState.zeros(1))
    s = 0.0
    for i in range(t):
        sk = s * k[i]
        s = al[i] * (s - be[i] * sk * k[i]) + be[i] * v[i] * k[i]
        assert out[i] == s * q[i]
    assert fin.s[0] == s


def test_orthonormal_keys_store_exactly():
    """alpha = beta = 1 with orthonormal keys: the delta rule writes each value
    exactly, S_T = sum v_t k_t^T, and o_t = v_t when q_t = k_t."""
    d = t = 8
    keys = np.eye(d)
    v = np.arange(t * d, dtype=np.float64).reshape(t, d) / 7.0
    inp = O.DeltaInputs(d, keys, keys, v, np.ones(t), np.ones(t), np.zeros(t, np.int64))
    out, fin = O.gated_delta_sequential(inp, O.DeltaState.zeros(d))
    assert np.array_equal(out.reshape(t, d), v)
    assert np.array_equal(fin.s.reshape(d, d), v.T)


def test_beta_zero_keeps_zero_state():
    inp = O.make_inputs(16, 4, segs_zero(16), 9)
    inp.beta[:] = 0.0
    out, fin = O.gated_delta_sequential(inp, O.DeltaState.zeros(4))
    assert not out.any() and not fin.s.any()


def test_sequential_ignores_init_like_reference():
    """delta.rs:137-141: prev_segment starts as None, so t = 0 resets."""
    inp = O.make_inputs(6, 3, segs_zero(6), 8)
    dirty = O.DeltaState(3, np.full(9, 5.0))
    a, sa = O.gated_delta_sequential(inp, O.DeltaState.zeros(3))
    b, sb = O.gated_delta_sequential(inp, dirty)
    assert np.array_equal(a, b) and np.array_equal(sa.s, sb.s)


# ---------------------------------------------------------------- transcription check

@pytest.mark.parametrize("t,d,segs,seed", [
    (40, 6, None, 2),
    (10, 4, [0, 0, 0, 1, 1, 2, 2, 2, 2, 3], 3),
    (17, 5, None, 11),
])
def test_c_oracle_bit_exact_vs_python_transcription(t, d, segs, seed):
    segs = segs or segs_zero(t)
    inp = O.make_inputs(t, d, segs, seed)
    out, fin = O.gated_delta_sequential(inp, O.DeltaState.zeros(d))
    pout, pfin = ref_python.sequential(d, list(inp.q), list(inp.k), list(inp.v),
                                       list(inp.alpha), list(inp.beta), segs, [0.0] * d * d)
    assert out.tolist() == pout
    assert fin.s.tolist() == pfin


def test_step_loop_honours_init_and_matches_steps():
    d, t = 4, 12
    inp = O.make_inputs(t, d, segs_zero(t), 21)
    init = O.DeltaState(d, O.make_normal(1, 22, d * d, 0.02))
    out, fin = O.gated_delta_step_loop(inp, init)
    s = init.clone()
    for i in range(t):
        o = O.gated_delta_step(s, inp.q[i * d:(i + 1) * d], inp.k[i * d:(i + 1) * d],
                               inp.v[i * d:(i + 1) * d], inp.alpha[i], inp.beta[i])
        assert np.array_equal(o, out[i * d:(i + 1) * d])
    assert np.array_equal(s.s, fin.s)


def test_batched_driver_matches_per_head():
    B, T, H, d = 2, 9, 3, 4
    q, k, v, al, be = O.make_qkv_gates(5, B * T, H, d)
    q, k, v = (x.reshape(B, T, H, d) for x in (q, k, v))
    al, be = al.reshape(B, T, H), be.reshape(B, T, H)
    o, so = O.gdr_dense(q, k, v, al, be, nthreads=3)
    for b in range(B):
        for h in range(H):
            inp = O.DeltaInputs(d, q[b, :, h], k[b, :, h], v[b, :, h], al[b, :, h], be[b, :, h])
            ro, rs = O.gated_delta_sequential(inp, O.DeltaState.zeros(d))
            assert np.array_equal(o[b, :, h].ravel(), ro)
            assert np.array_equal(so[b, h].ravel(), rs.s)


def test_generator_distributions():
    q, k, v, al, be = O.make_qkv_gates(3, 64, 2, 32)
    assert np.allclose(np.linalg.norm(q, axis=-1), 1.0)
    assert np.allclose(np.linalg.norm(k, axis=-1), 1.0)
    assert np.all((al > 0) & (al < 1)) and np.all((be > 0) & (be < 1))
    # alpha = exp(-softplus(x + 2)) with x ~ N(0,1): median exp(-softplus(2))
    assert abs(np.median(al) - math.exp(-math.log1p(math.exp(2.0)))) < 0.05


def _prep_python(cu, xq, xk, xv, bl, al, ah, w, b, cs, slots, zero_init, write_state, q_scale):
    """Pure-Python restatement of the input producer, one channel at a time
    with causal_conv1d_step (delta.rs:236-243) and l2norm/sigmoid/softplus
    (elementwise.rs), to check the batched C driver."""
    import math
    T, H, d = xq.shape
    outs = [np.zeros_like(xq) for _ in range(3)]
    alpha = np.zeros((T, H)); beta = np.zeros((T, H))
    cs = None if cs is None else cs.copy()
    for i in range(len(cu) - 1):
        slot = slots[i] if slots is not None else i
        valid = cs is not None and 0 <= slot < cs.shape[0]
        for h in range(H):
            for a, x in enumerate((xq, xk, xv)):
                for c in range(d):
                    st = np.zeros(3)
                    if valid and not zero_init:
                        st[:] = cs[slot, a, h, c]
                    for t in range(cu[i], cu[i + 1]):
                        outs[a][t, h, c] = O.causal_conv1d_step(st, w[a, h, c], x[t, h, c], b[a, h, c])
                    if valid and write_state:
                        cs[slot, a, h, c] = st
            for t in range(cu[i], cu[i + 1]):
                outs[0][t, h] = O.l2norm(outs[0][t, h], q_scale)
                outs[1][t, h] = O.l2norm(outs[1][t, h], 1.0)
                beta[t, h] = O.sigmoid(bl[t, h])
                alpha[t, h] = math.exp(-O.softplus(ah[h]) * O.softplus(al[t, h]))
    return outs[0], outs[1], outs[2], alpha, beta, cs


@pytest.mark.parametrize("zero_init,write_state", [(False, True), (True, True), (False, False)])
def test_prep_driver_matches_python_restatement(zero_init, write_state):
    rng = np.random.default_rng(5)
    H, d = 2, 8
    cu = np.array([0, 1, 3, 3, 9], dtype=np.int32)  # lengths 1, 2, 0, 6
    T = int(cu[-1])
    xq, xk, xv = (rng.normal(size=(T, H, d)) for _ in range(3))
    bl, al = rng.normal(size=(T, H)), rng.normal(size=(T, H))
    ah = rng.normal(size=H)
    w, b = rng.normal(size=(3, H, d, 4)), rng.normal(size=(3, H, d))
    cs = rng.normal(size=(6, 3, H, d, 3))
    slots = np.array([4, 0, 2, 9], dtype=np.int32)  # slot 9 is out of range
    got = O.gdr_prep(cu, xq, xk, xv, bl, al, ah, w, b, cs, slots, zero_init, write_state, 1.7)
    ref = _prep_python(cu, xq, xk, xv, bl, al, ah, w, b, cs, slots, zero_init, write_state, 1.7)
    for g, r in zip(got, ref):
        np.testing.assert_array_equal(g, r)
    if not write_state:
        np.testing.assert_array_equal(got[5], cs)


def test_groupnorm_heads_reference_cases():  # norm.rs:65-77, 117-130
    s = np.ones(4)
    a = O.groupnorm_heads(np.array([1.0, -2.0, 3.0, 0.5]).reshape(1, 1, 4), s, 1e-12)
    b = O.groupnorm_heads(np.array([10.0, -20.0, 30.0, 5.0]).reshape(1, 1, 4), s, 1e-12)
    assert np.max(np.abs(a - b)) < 1e-9
    y = O.groupnorm_heads(np.array([1.0, 1.0, 100.0, 100.0]).reshape(1, 2, 2), np.ones(2), 1e-12)
    assert np.max(np.abs(y.ravel()[:2] - y.ravel()[2:])) < 1e-9  # heads normalised independently


def test_groupnorm_heads_matches_numpy():
    rng = np.random.default_rng(3)
    x = rng.normal(size=(5, 3, 8))
    scale = rng.normal(size=24)  # only the first dh entries are used
    ref = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-6) * scale[:8]
    np.testing.assert_allclose(O.groupnorm_heads(x, scale, 1e-6), ref, rtol=1e-14, atol=1e-15)


def _loss(q, k, v, a, b, dO, dSf, seg, reset, init):
    """L = sum_t dO_t . o_t + <dS_final, S_T> through the step loop."""
    T, d = q.shape
    s = O.DeltaState(d, np.zeros(d * d) if init is None else init.ravel().copy())
    total = 0.0
    for t in range(T):
        if (t == 0 and reset) or (t > 0 and seg is not None and seg[t] != seg[t - 1]):
            s.s[:] = 0.0
        o = O.gated_delta_step(s, q[t], k[t], v[t], a[t], b[t])
        total += float(np.dot(dO[t], o))
    return total + float(np.dot(dSf.ravel(), s.s))


@pytest.mark.parametrize("reset,segmented", [(True, False), (True, True), (False, True)])
def test_backward_matches_central_differences(reset, segmented):
    """The adjoint against f64 central differences (gradcheck.rs: h = 1e-5,
    relative error against max(|fd|, |an|, 1e-6) at most 1e-6)."""
    rng = np.random.default_rng(7)
    T, d = 7, 3
    q, k, v, dO = (rng.normal(size=(T, d)) for _ in range(4))
    a = rng.uniform(0.3, 0.95, size=T)
    b = rng.uniform(0.1, 0.9, size=T)
    dSf = rng.normal(size=(d, d))
    init = rng.normal(size=(d, d))
    seg = np.array([0, 0, 1, 1, 1, 2, 2]) if segmented else None
    an = O.gated_delta_backward(q, k, v, a, b, dO, segment=seg, reset_at_start=reset, init=init,
                                d_state_final=dSf)
    params = [q, k, v, a, b, init]
    worst = 0.0
    for which, (x, g) in enumerate(zip(params, an)):
        for idx in np.ndindex(x.shape):
            xp = [p.copy() for p in params]; xm = [p.copy() for p in params]
            xp[which][idx] += 1e-5; xm[which][idx] -= 1e-5
            fd = (_loss(*xp[:5], dO, dSf, seg, reset, xp[5]) -
                  _loss(*xm[:5], dO, dSf, seg, reset, xm[5])) / 2e-5
            worst = max(worst, abs(fd - g[idx]) / max(abs(fd), abs(g[idx]), 1e-6))
    assert worst <= 1e-6, worst


@pytest.mark.parametrize("T,d,C", [(64, 8, 64), (130, 16, 64), (200, 32, 16)])
def test_chunked_backward_equals_sequential_adjoint(T, d, C):
    """The chunked (WY form) backward -- the per-chunk matrix products a
    tensor-core backward runs -- against the sequential adjoint, in f64."""
    from oracle import chunked_bwd as CB
    q, k, v, a, b = O.make_qkv_gates(7, T, 1, d)
    q, k, v, a, b = q[:, 0], k[:, 0], v[:, 0], a[:, 0], b[:, 0]
    rng = np.random.default_rng(T)
    dO = rng.normal(size=(T, d))
    dSf = rng.normal(size=(d, d))
    ref = O.gated_delta_backward(q, k, v, a, b, dO, d_state_final=dSf)
    got = CB.chunked_backward(q, k, v, a, b, dO, C, dSf)
    for x, y, name in zip(got, ref[:5], ("dq", "dk", "dv", "dalpha", "dbeta")):
        assert np.abs(x - y).max() <= 1e-11 * max(np.abs(y).max(), 1.0), name
    # and the chunked forward reproduces the sequential outputs and state
    o_seq, s_seq = O.gdr_dense(q[None, :, None], k[None, :, None], v[None, :, None],
                               a[None, :, None], b[None, :, None])
    S = np.zeros((d, d))
    outs = []
    for c in range(0, T, C):
        o_c, S, _ = CB.chunk_fwd(q[c:c + C], k[c:c + C], v[c:c + C], a[c:c + C], b[c:c + C], S)
        outs.append(o_c)
    assert np.abs(np.concatenate(outs) - o_seq[0, :, 0]).max() <= 1e-11
    assert np.abs(S - s_seq[0, 0]).max() <= 1e-11
