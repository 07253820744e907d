"""Host-side behaviour of the reference-shaped API (rhizome_b200.delta), no
GPU needed: DeltaInputs consistency as DeltaInputs::is_consistent states it
(crates/ops/src/delta.rs:46-55), shape errors raised before any device work,
the T = 0 case answered on the host (delta.rs:135), and DeltaState helpers
(delta.rs:59-90)."""
import numpy as np
import pytest

from rhizome_b200 import capi
from rhizome_b200 import delta as G


def _inputs(t, d, seg=None):
    rng = np.random.default_rng(t * 10 + d)
    seg = np.zeros(t, dtype=np.int64) if seg is None else np.asarray(seg)
    return G.DeltaInputs(d, rng.normal(size=t * d), rng.normal(size=t * d), rng.normal(size=t * d),
                         rng.random(t), rng.random(t), seg)


def test_consistency_rules():
    inp = _inputs(4, 3)
    assert inp.is_consistent() and not inp.is_empty() and len(inp) == 4
    # head_dim must be positive (delta.rs:50)
    zero_d = G.DeltaInputs(0, np.zeros(0), np.zeros(0), np.zeros(0), np.zeros(4), np.zeros(4),
                           np.zeros(4, dtype=np.int64))
    assert not zero_d.is_consistent()
    # q, k, v must hold T * d values; beta and segment T
    for field in ("q", "k", "v"):
        bad = _inputs(4, 3)
        setattr(bad, field, getattr(bad, field)[:-1])
        assert not bad.is_consistent(), field
    bad = _inputs(4, 3)
    bad.beta = bad.beta[:-1]
    assert not bad.is_consistent()
    bad = _inputs(4, 3)
    bad.segment = bad.segment[:-1]
    assert not bad.is_consistent()
    empty = _inputs(0, 3)
    assert empty.is_consistent() and empty.is_empty()


@pytest.mark.parametrize("entry", ["sequential", "scan_chunked", "multistep"])
def test_shape_errors_before_device_work(entry):
    bad = _inputs(5, 4)
    bad.k = bad.k[:-2]
    init = G.DeltaState.zeros(4)
    with pytest.raises(capi.ShapeError):
        if entry == "sequential":
            G.gated_delta_sequential(bad, init)
        elif entry == "scan_chunked":
            G.gated_delta_scan_chunked(bad, init, 8)
        else:
            G.gated_delta_multistep(bad, init, 3)


def test_step_shape_error_before_device_work():
    st = G.DeltaState.zeros(4)
    with pytest.raises(capi.ShapeError):
        G.gated_delta_step(st, np.zeros(4), np.zeros(3), np.zeros(4), 0.5, 0.5)
    with pytest.raises(capi.ShapeError):
        G.gated_delta_step(G.DeltaState(4, np.zeros(15)), np.zeros(4), np.zeros(4), np.zeros(4),
                           0.5, 0.5)


def test_empty_sequence_returns_the_initial_state_on_the_host():
    init = G.DeltaState(3, np.arange(9, dtype=np.float64))
    for fn in (lambda i: G.gated_delta_sequential(i, init),
               lambda i: G.gated_delta_scan_chunked(i, init, 64)):
        out, st = fn(_inputs(0, 3))
        assert out.size == 0 and np.array_equal(st.s, init.s)
        assert st is not init  # a clone, as init.clone() in the reference
    outs, states = G.gated_delta_multistep(_inputs(0, 3), init, 4)
    assert outs.size == 0 and states == []


def test_state_helpers():
    a = G.DeltaState.zeros(3)
    assert a.s.shape == (9,) and not a.s.any()
    b = a.clone()
    b.s[4] = -2.5
    assert a.max_abs_diff(b) == 2.5 and b.max_abs_diff(a) == 2.5
    assert not a.s.any()  # clone does not alias
    b.reset()
    assert not b.s.any() and a.max_abs_diff(b) == 0.0
