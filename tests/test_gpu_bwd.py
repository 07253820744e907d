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


# ---- the chunked tensor-core form (bf16, d = 128, no segments)

def bwd_form(name):
    import contextlib

    @contextlib.contextmanager
    def ctx():
        prev = ops.set_bwd_kernel(name)
        try:
            yield
        finally:
            ops.set_bwd_kernel(prev)
    return ctx()


def check_bf16_grads(got, ref, what):
    # fp16 products with fp32 accumulation: every output, dalpha and dbeta
    # included, is held to the bf16 bounds (relative and RMS-scaled)
    for g, r, n in zip(got, ref, NAMES):
        assert_bf16(g, r, f"{what} {n}", abs_bound=False)


@pytest.mark.parametrize("B,T,H,final_grad", [
    (1, 1, 1, False),      # one position, a one-row chunk
    (1, 64, 2, True),      # exactly one chunk
    (2, 130, 2, True),     # ragged last chunk of 2 positions
    (1, 257, 3, False),    # five chunks, last of one position
])
def test_tc_matches_adjoint_oracle(B, T, H, final_grad):
    inp = case(1000 + T, B, T, H, 128, "bf16", False, final_grad)
    with bwd_form("auto"):
        got = [host(x) for x in run_gpu("bf16", *inp)]
    check_bf16_grads(got, oracle_bwd(*inp), f"T={T}")


def test_tc_zero_alphas_exact_dalpha():
    """alpha = 0 at some positions (a full decay inside chunks and at a chunk
    start): dalpha there is finite and matches the adjoint; the division-free
    form needs no special case."""
    inp = list(case(77, 1, 192, 2, 128, "bf16", False, True))
    a = inp[3].copy()
    a[0, [5, 64, 100, 101, 191], :] = 0.0
    inp[3] = a
    with bwd_form("auto"):
        got = [host(x) for x in run_gpu("bf16", *inp)]
    check_bf16_grads(got, oracle_bwd(*inp), "zero alphas")


def test_tc_gradient_scale_invariance():
    """The upstream gradients enter scaled by an exact power of two: d_o and
    d_state_final multiplied by 2^-20 give the gradients multiplied by 2^-20
    (the same bits), far below fp16's normal range unscaled."""
    inp = list(case(33, 1, 130, 2, 128, "bf16", False, True))
    with bwd_form("auto"):
        a = [host(x) for x in run_gpu("bf16", *inp)]
        inp[5] = inp[5] * 2.0 ** -20
        inp[7] = inp[7] * 2.0 ** -20
        b = [host(x) for x in run_gpu("bf16", *inp)]
    for x, y, n in zip(a, b, NAMES):
        assert np.array_equal(x * 2.0 ** -20, y), n


def test_tc_agrees_with_scan_at_config_size():
    """configs[1] shape (B=4, T=4096, H=16): the tensor-core form against the
    fp32 reverse scan (itself pinned to the f64 adjoint above), same inputs."""
    B, T, H, d = 4, 4096, 16, 128
    g = torch.Generator(device="cuda").manual_seed(4096)
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(B, T, H, d, device="cuda", generator=g), dim=-1).to(torch.bfloat16)
    k = nrm(torch.randn(B, T, H, d, device="cuda", generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, H, d, device="cuda", generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, T, H, device="cuda", generator=g))
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, device="cuda", generator=g) + 2))
    d_o = torch.randn(B, T, H, d, device="cuda", generator=g).to(torch.bfloat16)
    dsf = torch.randn(B, H, d, d, device="cuda", generator=g) * 0.1
    with bwd_form("auto"):
        tc = [host(x) for x in ops.gdr_scan_chunked_bwd(q, k, v, alpha, beta, d_o, d_state_final=dsf)]
    with bwd_form("scan"):
        sc = [host(x) for x in ops.gdr_scan_chunked_bwd(q, k, v, alpha, beta, d_o, d_state_final=dsf)]
    check_bf16_grads(tc, sc, "configs[1]")


def test_tc_deterministic():
    inp = case(21, 2, 200, 2, 128, "bf16", False, True)
    with bwd_form("auto"):
        a = [host(x) for x in run_gpu("bf16", *inp)]
        b = [host(x) for x in run_gpu("bf16", *inp)]
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
