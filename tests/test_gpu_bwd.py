"""GPU parity of the scan's backward (rhz_gdr_scan_chunked_bwd) against the
f64 adjoint oracle (oracle/gdr_oracle.c rhzo_gated_delta_backward, itself
checked against f64 central differences in tests/test_oracle.py)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from rhizome_b200 import ops
from tests.gpu_util import host, make_inputs, to_dev
from tests.tolerance import assert_bf16, bf16_round, error_stats

pytestmark = pytest.mark.gpu


def f32(x):
    return np.asarray(x, dtype=np.float64).astype(np.float32).astype(np.float64)


def oracle_bwd(q, k, v, a, b, dO, seg, dSf):
    B, T, H, d = q.shape
    outs = [np.zeros_like(q), np.zeros_like(q), np.zeros_like(q), np.zeros_like(a), np.zeros_like(b)]
    for bi in range(B):
        for h in range(H):
            r = O.gated_delta_backward(q[bi, :, h], k[bi, :, h], v[bi, :, h], a[bi, :, h],
                                       b[bi, :, h], dO[bi, :, h],
                                       segment=None if seg is None else seg[bi],
                                       reset_at_start=True,
                                       d_state_final=None if dSf is None else dSf[bi, h])
            for o, x in zip(outs[:3], r[:3]):
                o[bi, :, h] = x
            outs[3][bi, :, h] = r[3]
            outs[4][bi, :, h] = r[4]
    return outs


def case(seed, B, T, H, d, dtype, segmented, final_grad):
    rng = np.random.default_rng(seed)
    q, k, v, a, b = (x.reshape((B, T, H) + x.shape[2:]) for x in make_inputs(seed, B * T, H, d, dtype))
    rnd = bf16_round if dtype == "bf16" else f32
    dO = rnd(rng.normal(size=(B, T, H, d)))
    seg = np.cumsum(rng.random((B, T)) < 0.05, axis=1).astype(np.int64) if segmented else None
    dSf = f32(rng.normal(size=(B, H, d, d))) if final_grad else None
    return q, k, v, a, b, dO, seg, dSf


def run_gpu(dtype, q, k, v, a, b, dO, seg, dSf):
    td = torch.bfloat16 if dtype == "bf16" else torch.float32
    return ops.gdr_scan_chunked_bwd(to_dev(q, td), to_dev(k, td), to_dev(v, td),
                                    to_dev(a, torch.float32), to_dev(b, torch.float32),
                                    to_dev(dO, td),
                                    segment=None if seg is None else to_dev(seg, torch.int64),
                                    d_state_final=None if dSf is None else to_dev(dSf, torch.float32))


NAMES = ("dq", "dk", "dv", "dalpha", "dbeta")


@pytest.mark.parametrize("B,T,H,d,segmented,final_grad", [
    (1, 1, 1, 16, False, False),
    (2, 7, 2, 32, True, True),
    (2, 37, 2, 64, False, True),
    (1, 200, 2, 128, True, False),
    (2, 129, 3, 128, True, True),
])
def test_f32_matches_adjoint_oracle(B, T, H, d, segmented, final_grad):
    inp = case(T * d, B, T, H, d, "f32", segmented, final_grad)
    got = [host(x) for x in run_gpu("f32", *inp)]
    ref = oracle_bwd(*inp)
    for g, r, n in zip(got, ref, NAMES):
        st = error_stats(g, r)
        # fp32 over a T-step reverse scan against f64, in the benchmark's form
        # (max error relative to max |ref|)
        assert st["finite"] and st["max_rel"] <= 1e-5, (n, st)


def test_bf16_inputs():
    inp = case(5, 2, 130, 2, 128, "bf16", True, True)
    got = [host(x) for x in run_gpu("bf16", *inp)]
    ref = oracle_bwd(*inp)
    for g, r, n in zip(got, ref, NAMES):
        if n in ("dalpha", "dbeta"):
            st = error_stats(g, r)  # f32 outputs: only the inputs were bf16
            assert st["finite"] and st["max_rel"] <= 1e-5, (n, st)
        else:
            # gradients of O(1-10) magnitude: one bf16 rounding of the output
            # alone exceeds a fixed 1e-2 cap, so the relative and RMS-scaled
            # bounds apply (as for other outputs that are not O(0.1))
            assert_bf16(g, r, n, abs_bound=False)


def test_deterministic():
    inp = case(9, 2, 64, 2, 128, "f32", True, True)
    a = [host(x) for x in run_gpu("f32", *inp)]
    b = [host(x) for x in run_gpu("f32", *inp)]
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
