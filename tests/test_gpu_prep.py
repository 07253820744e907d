"""GPU parity of the Local block's input producer (rhz_gdr_prep) against the
f64 oracle (oracle/gdr_oracle.c rhzo_gdr_prep, itself checked against a
pure-Python restatement of causal_conv1d_step / l2norm / sigmoid / softplus):
conv carried per sequence from slots, norms, gates, dense and packed batches,
decode continuity, and prep followed by the recurrence."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from rhizome_b200 import ops
from tests.gpu_util import host, to_dev
from tests.tolerance import assert_bf16, assert_fp32, bf16_round

pytestmark = pytest.mark.gpu

TD = {"f32": torch.float32, "bf16": torch.bfloat16}


def f32(x):
    return np.asarray(x, dtype=np.float64).astype(np.float32).astype(np.float64)


def params(rng, H, d):
    return f32(rng.normal(size=H)), f32(rng.normal(scale=0.5, size=(3, H, d, 4))), \
        f32(rng.normal(scale=0.1, size=(3, H, d)))


def raw(rng, T, H, d, dtype):
    rnd = bf16_round if dtype == "bf16" else f32
    xs = [rnd(rng.normal(size=(T, H, d))) for _ in range(3)]
    return xs + [f32(rng.normal(size=(T, H))), f32(rng.normal(scale=2.0, size=(T, H)))]


def gpu_prep(dtype, xs, bl, al, ah, w, b, cs=None, slots=None, cu=None, dense=None, **kw):
    """Run the producer on the device; returns host arrays in the packed
    layout ([tokens, H, d] and [tokens, H]) and the conv state after."""
    td = TD[dtype]
    shape = dense if dense is not None else xs[0].shape
    H, d = shape[-2], shape[-1]
    X = [to_dev(x.reshape(shape), td) for x in xs]
    dev_cs = None if cs is None else to_dev(cs, torch.float32)
    out = ops.gdr_prep(*X, to_dev(bl.reshape(shape[:-1]), torch.float32),
                       to_dev(al.reshape(shape[:-1]), torch.float32), to_dev(ah, torch.float32),
                       to_dev(w, torch.float32), to_dev(b, torch.float32), conv_state=dev_cs,
                       slot_idx=None if slots is None else to_dev(slots, torch.int32),
                       cu_seqlens=None if cu is None else to_dev(cu, torch.int32), **kw)
    q, k, v = (host(t).reshape(-1, H, d) for t in out[:3])
    a, bt = (host(t).reshape(-1, H) for t in out[3:])
    return q, k, v, a, bt, (None if dev_cs is None else host(dev_cs))


def check(dtype, got, ref, what):
    names = ("q", "k", "v", "alpha", "beta")
    for g, r, n in zip(got[:5], ref[:5], names):
        if dtype == "f32" or n in ("alpha", "beta"):
            assert_fp32(g, r, f"{what} {n}")
        else:
            # f32 arithmetic, one bf16 rounding of the result
            bad = np.abs(g - r) > 2.0 ** -8 * np.abs(r) + 1e-6
            assert not bad.any(), f"{what} {n}: {bad.sum()} elements beyond one bf16 rounding"
    if ref[5] is not None:
        np.testing.assert_array_equal(got[5], ref[5], err_msg=f"{what} conv state")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_dense_matches_oracle(dtype):
    rng = np.random.default_rng(11)
    B, T, H, d = 3, 37, 4, 128
    xs_bl_al = raw(rng, B * T, H, d, dtype)
    xs, bl, al = xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4]
    ah, w, b = params(rng, H, d)
    cs = f32(rng.normal(size=(B, 3, H, d, 3)))
    cu = np.arange(B + 1, dtype=np.int32) * T
    q_scale = math.sqrt(d)
    ref = O.gdr_prep(cu, *xs, bl, al, ah, w, b, cs, None, False, True, f32(q_scale))
    got = gpu_prep(dtype, xs, bl, al, ah, w, b, cs=cs, dense=(B, T, H, d), q_scale=q_scale)
    check(dtype, got, ref, "dense")


@pytest.mark.parametrize("zero_init,write_state", [(False, True), (True, True), (False, False)])
def test_packed_with_slots(zero_init, write_state):
    rng = np.random.default_rng(12)
    H, d = 3, 64
    lens = np.array([1, 2, 0, 5, 64, 3, 130])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    xs_bl_al = raw(rng, int(cu[-1]), H, d, "f32")
    xs, bl, al = xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4]
    ah, w, b = params(rng, H, d)
    cs = f32(rng.normal(size=(10, 3, H, d, 3)))
    slots = np.array([7, 2, 9, 0, 4, 11, 5], dtype=np.int32)  # 11 is out of range
    ref = O.gdr_prep(cu, *xs, bl, al, ah, w, b, cs, slots, zero_init, write_state, 1.0)
    got = gpu_prep("f32", xs, bl, al, ah, w, b, cs=cs, slots=slots, cu=cu, zero_init=zero_init,
                   write_state=write_state)
    check("f32", got, ref, "packed")


@pytest.mark.parametrize("d", [4, 64, 256, 512])
def test_head_widths(d):
    rng = np.random.default_rng(d)
    H = 2
    cu = np.array([0, 5, 9], dtype=np.int32)
    xs_bl_al = raw(rng, 9, H, d, "f32")
    ah, w, b = params(rng, H, d)
    ref = O.gdr_prep(cu, *xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4], ah, w, b, None, None, False,
                     True, 2.0)
    got = gpu_prep("f32", xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4], ah, w, b, cu=cu, q_scale=2.0)
    check("f32", got, ref, f"d={d}")


def test_decode_steps_continue_the_sequence():
    """Token-by-token calls (one token per sequence, state carried in the
    slots) give what one call over the whole sequences gives."""
    rng = np.random.default_rng(13)
    n, steps, H, d = 6, 5, 4, 128
    xs_bl_al = raw(rng, n * steps, H, d, "f32")
    xs = [x.reshape(n, steps, H, d) for x in xs_bl_al[:3]]
    bl, al = (x.reshape(n, steps, H) for x in xs_bl_al[3:])
    ah, w, b = params(rng, H, d)
    cs0 = f32(rng.normal(size=(8, 3, H, d, 3)))
    slots = np.array([3, 0, 7, 1, 5, 2], dtype=np.int32)
    cu = np.arange(n + 1, dtype=np.int32) * steps
    ref = O.gdr_prep(cu, *[x.reshape(-1, H, d) for x in xs], bl.reshape(-1, H), al.reshape(-1, H),
                     ah, w, b, cs0, slots, False, True, 1.5)
    dev_cs = to_dev(cs0, torch.float32)
    outs = []
    for t in range(steps):
        step = [np.ascontiguousarray(x[:, t]) for x in xs]
        X = [to_dev(x, torch.float32) for x in step]
        o = ops.gdr_prep(*X, to_dev(np.ascontiguousarray(bl[:, t]), torch.float32),
                         to_dev(np.ascontiguousarray(al[:, t]), torch.float32),
                         to_dev(ah, torch.float32), to_dev(w, torch.float32),
                         to_dev(b, torch.float32), conv_state=dev_cs,
                         slot_idx=to_dev(slots, torch.int32),
                         cu_seqlens=to_dev(np.arange(n + 1, dtype=np.int32), torch.int32),
                         q_scale=1.5)
        outs.append([host(z) for z in o])
    for i, name in enumerate(("q", "k", "v")):
        got = np.stack([outs[t][i] for t in range(steps)], axis=1).reshape(-1, H, d)
        assert_fp32(got, ref[i], f"decode {name}")
    np.testing.assert_array_equal(host(dev_cs), ref[5])


def test_config_size_bf16():
    """configs[1] shape (B=4, T=4096, H=16, d=128) through the producer."""
    rng = np.random.default_rng(14)
    B, T, H, d = 4, 4096, 16, 128
    xs_bl_al = raw(rng, B * T, H, d, "bf16")
    ah, w, b = params(rng, H, d)
    cs = f32(rng.normal(size=(B, 3, H, d, 3)))
    cu = np.arange(B + 1, dtype=np.int32) * T
    ref = O.gdr_prep(cu, *xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4], ah, w, b, cs, None, False, True,
                     math.sqrt(d))
    got = gpu_prep("bf16", xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4], ah, w, b, cs=cs,
                   dense=(B, T, H, d), q_scale=math.sqrt(d))
    check("bf16", got, ref, "configs[1] size")


def test_prep_then_recurrence_matches_oracle():
    """Raw projections -> producer -> packed recurrence from slot states, on
    the device and in f64."""
    rng = np.random.default_rng(15)
    H, d = 4, 128
    lens = np.array([70, 1, 129, 3])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tokens = int(cu[-1])
    xs_bl_al = raw(rng, tokens, H, d, "bf16")
    ah, w, b = params(rng, H, d)
    cs = f32(rng.normal(size=(4, 3, H, d, 3)))
    slots = np.array([2, 0, 3, 1], dtype=np.int32)
    pool = f32(rng.normal(scale=0.02, size=(4, H, d, d)))
    rq, rk, rv, ra, rb, _ = O.gdr_prep(cu, *xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4], ah, w, b, cs,
                                       slots, False, True, 1.0)
    # The recurrence receives what the device producer hands it: bf16 q/k/v,
    # f32 gates.
    ro, rpool = O.gdr_varlen(cu, bf16_round(rq), bf16_round(rk), bf16_round(rv), f32(ra), f32(rb),
                             state_in=pool, state_in_index=slots, state_out_index=slots)
    X = [to_dev(x, torch.bfloat16) for x in xs_bl_al[:3]]
    q, k, v, a, bt = ops.gdr_prep(*X, to_dev(xs_bl_al[3], torch.float32),
                                  to_dev(xs_bl_al[4], torch.float32), to_dev(ah, torch.float32),
                                  to_dev(w, torch.float32), to_dev(b, torch.float32),
                                  conv_state=to_dev(cs, torch.float32),
                                  slot_idx=to_dev(slots, torch.int32),
                                  cu_seqlens=to_dev(cu, torch.int32))
    dpool = to_dev(pool, torch.float32)
    o = ops.gdr_varlen_fwd(q, k, v, a, bt, to_dev(cu, torch.int32), dpool,
                           slot_idx=to_dev(slots, torch.int32))
    torch.cuda.synchronize()
    assert_bf16(host(o), ro, "prep -> recurrence o")
    assert_bf16(host(dpool), rpool, "prep -> recurrence states")


def test_inputs_on_8_byte_boundaries():
    """bf16 inputs that start 8 bytes past a 16-byte boundary (all the C ABI
    asks of bf16 arrays) take the form with 8-byte loads and give the same
    answer as aligned inputs, within one bf16 rounding of the oracle."""
    rng = np.random.default_rng(16)
    H, d = 4, 128
    lens = np.array([70, 1, 129, 3])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tokens = int(cu[-1])
    xs_bl_al = raw(rng, tokens, H, d, "bf16")
    ah, w, b = params(rng, H, d)
    cs = f32(rng.normal(size=(4, 3, H, d, 3)))
    slots = np.array([2, 0, 3, 1], dtype=np.int32)
    ref = O.gdr_prep(cu, *xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4], ah, w, b, cs, slots, False, True,
                     math.sqrt(d))
    X = []
    for x in xs_bl_al[:3]:
        buf = torch.empty(tokens * H * d + 4, dtype=torch.bfloat16, device="cuda")
        view = buf[4:].view(tokens, H, d)
        view.copy_(to_dev(x, torch.bfloat16))
        assert view.data_ptr() % 16 == 8
        X.append(view)
    dev_cs = to_dev(cs, torch.float32)
    out = ops.gdr_prep(*X, to_dev(xs_bl_al[3], torch.float32), to_dev(xs_bl_al[4], torch.float32),
                       to_dev(ah, torch.float32), to_dev(w, torch.float32), to_dev(b, torch.float32),
                       conv_state=dev_cs, slot_idx=to_dev(slots, torch.int32),
                       cu_seqlens=to_dev(cu, torch.int32), q_scale=math.sqrt(d))
    got = [host(t) for t in out] + [host(dev_cs)]
    check("bf16", got, ref, "8-byte boundaries")


def test_rows_outside_sequences_bf16_d128():
    """A packed stream whose offsets leave rows before the first sequence and
    after the last uncovered, with an empty sequence and sequences that start
    and end inside 64-token tiles: covered rows match the oracle, uncovered
    rows of the outputs are left as they were."""
    from rhizome_b200 import capi
    rng = np.random.default_rng(17)
    H, d = 3, 128
    tokens = 300
    cu = np.array([5, 69, 69, 70, 133, 200, 293], dtype=np.int32)
    xs_bl_al = raw(rng, tokens, H, d, "bf16")
    ah, w, b = params(rng, H, d)
    cs = f32(rng.normal(size=(7, 3, H, d, 3)))
    slots = np.array([6, 1, 0, 3, 2, 5], dtype=np.int32)
    ref = O.gdr_prep(cu, *xs_bl_al[:3], xs_bl_al[3], xs_bl_al[4], ah, w, b, cs, slots, False, True,
                     1.0)
    X = [to_dev(x, torch.bfloat16) for x in xs_bl_al[:3]]
    dev_cs = to_dev(cs, torch.float32)
    sentinel = -7.0
    outs = [torch.full((tokens, H, d), sentinel, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    outs += [torch.full((tokens, H), sentinel, dtype=torch.float32, device="cuda") for _ in range(2)]
    # every device argument stays referenced until the call has run
    args = [to_dev(xs_bl_al[3], torch.float32), to_dev(xs_bl_al[4], torch.float32),
            to_dev(ah, torch.float32), to_dev(w, torch.float32), to_dev(b, torch.float32), dev_cs,
            to_dev(slots, torch.int32), to_dev(cu, torch.int32)]
    capi.call("rhz_gdr_prep", *[t.data_ptr() for t in outs], *[t.data_ptr() for t in X],
              *[t.data_ptr() for t in args], len(slots), 0, tokens, 7, H, d, 1.0,
              capi.RHZ_DTYPE_BF16, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = [host(t) for t in outs] + [host(dev_cs)]
    inside = np.zeros(tokens, dtype=bool)
    inside[cu[0]:cu[-1]] = True
    for g in got[:5]:
        assert np.all(g[~inside] == sentinel), "an uncovered row was written"
    check("bf16", [g[inside] for g in got[:5]] + [got[5]], [r[inside] for r in ref[:5]] + [ref[5]],
          "uncovered rows")
