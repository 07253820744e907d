"""GPU parity of the per-head output norm (groupnorm_heads, norm.rs:48-60):
the standalone kernel and the norm fused into the recurrence's epilogue,
against the f64 oracle (itself pinned to the reference's norm tests)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from rhizome_b200 import ops
from tests.gpu_util import chunk_form, host, make_inputs, to_dev
from tests.tolerance import assert_bf16, assert_fp32, bf16_round, error_stats

pytestmark = pytest.mark.gpu


def f32(x):
    return np.asarray(x, dtype=np.float64).astype(np.float32).astype(np.float64)


@pytest.mark.parametrize("d", [4, 64, 128, 256, 512])
def test_standalone_f32(d):
    rng = np.random.default_rng(d)
    rows, H = 37, 3
    x = f32(rng.normal(scale=3.0, size=(rows, H, d)))
    scale = f32(rng.normal(size=H * d))  # only scale[:d] is used, as in the reference
    ref = O.groupnorm_heads(x, scale, 1e-6)
    got = ops.groupnorm_heads(to_dev(x, torch.float32), to_dev(scale, torch.float32), eps=1e-6)
    assert_fp32(host(got), ref, f"groupnorm d={d}")


def test_standalone_bf16_in_place():
    rng = np.random.default_rng(1)
    rows, H, d = 1000, 16, 128
    x = bf16_round(rng.normal(size=(rows, H, d)))
    scale = f32(rng.normal(size=d))
    ref = O.groupnorm_heads(x, scale, 1e-5)
    dx = to_dev(x, torch.bfloat16)
    ops.groupnorm_heads(dx, to_dev(scale, torch.float32), eps=1e-5, out=dx)
    got = host(dx)
    bad = np.abs(got - ref) > 2.0 ** -8 * np.abs(ref) + 1e-6
    assert not bad.any(), f"{bad.sum()} elements beyond one bf16 rounding"


def _varlen_case(dtype, seed):
    rng = np.random.default_rng(seed)
    H, d = 4, 128
    lens = np.array([130, 1, 64, 0, 200])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    q, k, v, a, b = make_inputs(seed, int(cu[-1]), H, d, dtype)
    pool = f32(rng.normal(scale=0.02, size=(6, H, d, d)))
    slots = np.array([5, 0, 3, 1, 2], dtype=np.int32)
    scale = f32(rng.normal(size=d))
    return cu, q, k, v, a, b, pool, slots, scale


@pytest.mark.parametrize("form", ["pair", "solo"])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_varlen_with_output_norm_matches_oracle(dtype, form):
    if dtype == "f32" and form == "solo":
        pytest.skip("the f32 path does not use the tensor-core kernels")
    with chunk_form(form):
        _check_varlen_with_output_norm(dtype)


def _check_varlen_with_output_norm(dtype):
    cu, q, k, v, a, b, pool, slots, scale = _varlen_case(dtype, 21)
    td = torch.bfloat16 if dtype == "bf16" else torch.float32
    dpool = to_dev(pool, torch.float32)
    o = ops.gdr_varlen_fwd_norm(to_dev(q, td), to_dev(k, td), to_dev(v, td),
                                to_dev(a, torch.float32), to_dev(b, torch.float32),
                                to_dev(cu, torch.int32), to_dev(scale, torch.float32), 1e-6,
                                state_pool=dpool, slot_idx=to_dev(slots, torch.int32))
    torch.cuda.synchronize()
    ro, rpool = O.gdr_varlen(cu, q, k, v, a, b, state_in=pool, state_in_index=slots,
                             state_out_index=slots)
    rn = O.groupnorm_heads(ro, scale, 1e-6)
    if dtype == "bf16":
        # normalised rows are O(1): the relative and RMS-scaled bounds apply
        assert_bf16(host(o), rn, "normed o", abs_bound=False)
        assert_bf16(host(dpool), rpool, "states")
    else:
        # The composition against f64 end to end, in the benchmark's form
        # (max relative error against max |ref|) ...
        st = error_stats(host(o), rn)
        assert st["finite"] and st["max_rel"] <= 1e-5, st
        assert_fp32(host(dpool), rpool, "states")
        # ... and the norm op itself at its own elementwise tolerance
        # (docs/kernels.md rmsnorm row), given the device recurrence's output.
        plain = ops.gdr_varlen_fwd(to_dev(q, td), to_dev(k, td), to_dev(v, td),
                                   to_dev(a, torch.float32), to_dev(b, torch.float32),
                                   to_dev(cu, torch.int32), state_pool=to_dev(pool, torch.float32),
                                   slot_idx=to_dev(slots, torch.int32))
        assert_fp32(host(o), O.groupnorm_heads(host(plain), scale, 1e-6), "norm op")


@pytest.mark.parametrize("form", ["pair", "solo"])
def test_fused_epilogue_equals_separate_norm(form):
    """bf16: the norm in the recurrence epilogue (on the fp32 accumulator)
    against recurrence -> bf16 o -> standalone norm: within one extra bf16
    rounding of each other."""
    with chunk_form(form):
        _check_fused_epilogue()


def _check_fused_epilogue():
    cu, q, k, v, a, b, pool, slots, scale = _varlen_case("bf16", 22)
    args = [to_dev(x, torch.bfloat16) for x in (q, k, v)] + \
        [to_dev(a, torch.float32), to_dev(b, torch.float32), to_dev(cu, torch.int32)]
    s = to_dev(scale, torch.float32)
    fused = ops.gdr_varlen_fwd_norm(*args, s, 1e-6, state_pool=to_dev(pool, torch.float32),
                                    slot_idx=to_dev(slots, torch.int32))
    plain = ops.gdr_varlen_fwd(*args, state_pool=to_dev(pool, torch.float32),
                               slot_idx=to_dev(slots, torch.int32))
    sep = ops.groupnorm_heads(plain, s, eps=1e-6)
    f, g = host(fused), host(sep)
    bad = np.abs(f - g) > 2.0 ** -6 * np.abs(g) + 1e-3
    assert not bad.any(), f"{bad.sum()} elements differ by more than two bf16 roundings"
