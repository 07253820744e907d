"""The reference's own GDR tests (crates/ops/src/delta.rs:245-369), run on
the GPU through the reference-shaped API (rhizome_b200.delta), each result
also checked against the f64 oracle at the fp32 tolerance."""
import numpy as np
import pytest

from oracle import oracle as O
from rhizome_b200 import capi
from rhizome_b200 import delta as G
from tests.tolerance import assert_fp32

pytestmark = pytest.mark.gpu


def inputs(t, d, segs, seed):
    o = O.make_inputs(t, d, segs, seed)
    return G.DeltaInputs(d, o.q, o.k, o.v, o.alpha, o.beta, o.segment), o


def test_inputs_validate_shapes():
    inp, _ = inputs(4, 3, [0, 0, 0, 0], 1)
    assert inp.is_consistent() and not inp.is_empty()
    bad = G.DeltaInputs(3, inp.q[:-1], inp.k, inp.v, inp.alpha, inp.beta, inp.segment)
    with pytest.raises(capi.ShapeError):
        G.gated_delta_sequential(bad, G.DeltaState.zeros(3))


def test_chunked_matches_sequential_single_segment():
    t, d = 40, 6
    inp, oinp = inputs(t, d, [0] * t, 2)
    init = G.DeltaState.zeros(d)
    a, sa = G.gated_delta_sequential(inp, init)
    ra, rsa = O.gated_delta_sequential(oinp, O.DeltaState.zeros(d))
    assert_fp32(a, ra, "sequential")
    assert_fp32(sa.s, rsa.s, "sequential state")
    for chunk in [1, 3, 8, 64]:
        b, sb = G.gated_delta_scan_chunked(inp, init, chunk)
        assert np.all(np.abs(a - b) < 1e-10), chunk
        assert sa.max_abs_diff(sb) < 1e-10


def test_chunked_matches_sequential_with_segments():
    d = 4
    segs = [0, 0, 0, 1, 1, 2, 2, 2, 2, 3]
    inp, oinp = inputs(len(segs), d, segs, 3)
    init = G.DeltaState.zeros(d)
    a, sa = G.gated_delta_sequential(inp, init)
    b, sb = G.gated_delta_scan_chunked(inp, init, 4)
    assert np.all(np.abs(a - b) < 1e-10)
    assert sa.max_abs_diff(sb) < 1e-10
    ra, rsa = O.gated_delta_sequential(oinp, O.DeltaState.zeros(d))
    assert_fp32(a, ra, "segments")
    assert_fp32(sa.s, rsa.s, "segments state")


def test_multistep_matches_repeated_step():
    d, t = 5, 8
    inp, oinp = inputs(t, d, [0] * t, 4)
    init = G.DeltaState.zeros(d)
    outs, states = G.gated_delta_multistep(inp, init, 8)
    seq, final_state = G.gated_delta_sequential(inp, init)
    assert_fp32(outs, seq, "multistep vs sequential")
    assert states[t - 1].max_abs_diff(final_state) < 1e-6
    routs, rstates = O.gated_delta_multistep(oinp, O.DeltaState.zeros(d), 8)
    assert_fp32(outs, routs, "multistep vs oracle")
    for s, r in zip(states, rstates):
        assert_fp32(s.s, r.s, "multistep states")


def test_segment_reset_makes_history_irrelevant():
    d = 3
    inp, _ = inputs(4, d, [0, 0, 1, 1], 5)
    dirty = G.DeltaState.zeros(d)
    dirty.s[:] = 3.0
    a, _ = G.gated_delta_sequential(inp, G.DeltaState.zeros(d))
    b, _ = G.gated_delta_sequential(inp, dirty)
    for i in range(2 * d, 4 * d):
        assert abs(a[i] - b[i]) < 1e-12


def test_alpha_zero_forgets_the_past():
    d = 3
    s = G.DeltaState.zeros(d)
    s.s[:] = 1.0
    o = G.gated_delta_step(s, [1.0, 1.0, 1.0], [1.0, 0.0, 0.0], [0.0, 0.0, 0.0], 0.0, 0.5)
    assert np.all(np.abs(o) < 1e-12)


def test_step_matches_oracle_step():
    d = 32
    _, oinp = inputs(1, d, [0], 12)
    init = O.make_normal(2, 22, d * d, 0.3)
    s = G.DeltaState(d, init.copy())
    rs = O.DeltaState(d, init.copy())
    o = G.gated_delta_step(s, oinp.q, oinp.k, oinp.v, oinp.alpha[0], oinp.beta[0])
    ro = O.gated_delta_step(rs, oinp.q, oinp.k, oinp.v, oinp.alpha[0], oinp.beta[0])
    assert_fp32(o, ro, "step o")
    assert_fp32(s.s, rs.s, "step state")
