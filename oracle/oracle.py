"""ctypes wrapper over oracle/gdr_oracle.c -- test infrastructure only.

Mirrors the reference's Rust API (crates/ops/src/delta.rs, rng.rs,
elementwise.rs) on numpy f64 arrays so tests read like the reference's own.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np

from . import build as _build

_lib = None

_dp = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_ip = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_up = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = C.CDLL(path)
        i64, u64, d64 = C.c_int64, C.c_uint64, C.c_double
        L.rhzo_philox_fill_u32.argtypes = [u64, u64, u64, _up]
        L.rhzo_philox_fill_f64.argtypes = [u64, u64, u64, _dp]
        L.rhzo_philox_fill_normal.argtypes = [u64, u64, u64, _dp]
        L.rhzo_philox_block_raw.argtypes = [C.c_uint32, C.c_uint32, u64, u64, _up]
        L.rhzo_stateless_uniform.argtypes = [u64, u64, u64]
        L.rhzo_stateless_uniform.restype = d64
        L.rhzo_sigmoid.argtypes = [d64]
        L.rhzo_sigmoid.restype = d64
        L.rhzo_softplus.argtypes = [d64]
        L.rhzo_softplus.restype = d64
        L.rhzo_l2norm.argtypes = [_dp, i64, d64, _dp]
        L.rhzo_gated_delta_step.argtypes = [_dp, i64, _dp, _dp, _dp, d64, d64, _dp]
        L.rhzo_inputs_consistent.argtypes = [i64] * 7
        L.rhzo_inputs_consistent.restype = C.c_int
        L.rhzo_gated_delta_sequential.argtypes = [i64, i64, _dp, _dp, _dp, _dp, _dp, _ip, _dp,
                                                  _dp, _dp]
        L.rhzo_gated_delta_scan_chunked.argtypes = [i64, i64, _dp, _dp, _dp, _dp, _dp, _ip,
                                                    _dp, i64, _dp, _dp]
        L.rhzo_gated_delta_multistep.argtypes = [i64, i64, _dp, _dp, _dp, _dp, _dp, _ip, _dp,
                                                 i64, _dp, _dp]
        L.rhzo_gated_delta_multistep.restype = i64
        L.rhzo_causal_conv1d_step.argtypes = [_dp, _dp, d64, d64]
        L.rhzo_causal_conv1d_step.restype = d64
        L.rhzo_gated_delta_step_loop.argtypes = [i64, i64, _dp, _dp, _dp, _dp, _dp, _dp, _dp,
                                                 _dp]
        vp = C.c_void_p
        L.rhzo_gdr_varlen.argtypes = [i64, _ip, i64, i64, _dp, _dp, _dp, _dp, _dp, vp, vp,
                                      _dp, vp, vp, C.c_int]
        L.rhzo_gdr_dense.argtypes = [i64, i64, i64, i64, _dp, _dp, _dp, _dp, _dp, vp, _dp, vp,
                                     C.c_int]
        L.rhzo_make_qkv_gates.argtypes = [u64, i64, i64, i64, _dp, _dp, _dp, _dp, _dp]
        L.rhzo_make_normal.argtypes = [u64, u64, i64, d64, _dp]
        L.rhzo_make_test_inputs.argtypes = [i64, i64, u64, _dp, _dp, _dp, _dp, _dp]
        _i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
        L.rhzo_gdr_prep.argtypes = [i64, _i32p, i64, i64, _dp, _dp, _dp, _dp, _dp, _dp, _dp,
                                    _dp, vp, vp, i64, C.c_int, C.c_int, d64, _dp, _dp, _dp,
                                    _dp, _dp]
        L.rhzo_groupnorm_heads.argtypes = [_dp, i64, i64, i64, _dp, d64, _dp]
        L.rhzo_gated_delta_backward.argtypes = [i64, i64, _dp, _dp, _dp, _dp, _dp, vp, C.c_int,
                                                vp, _dp, vp, _dp, _dp, _dp, _dp, _dp, vp]
        _lib = L
    return _lib


def _f64(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float64)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ----------------------------------------------------------------------------
# crates/ops/src/rng.rs
# ----------------------------------------------------------------------------

class Philox:
    """Philox-4x32-10 (crates/ops/src/rng.rs:14-97), bulk draws via the C port."""

    def __init__(self, seed: int, stream: int):
        self.seed, self.stream = int(seed), int(stream)

    def u32(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint32)
        lib().rhzo_philox_fill_u32(self.seed, self.stream, n, out)
        return out

    def f64(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float64)
        lib().rhzo_philox_fill_f64(self.seed, self.stream, n, out)
        return out

    def normal(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float64)
        lib().rhzo_philox_fill_normal(self.seed, self.stream, n, out)
        return out


def philox_block(key0: int, key1: int, counter: int, stream: int) -> np.ndarray:
    out = np.empty(4, dtype=np.uint32)
    lib().rhzo_philox_block_raw(key0, key1, counter, stream, out)
    return out


def stateless_uniform(seed: int, stream: int, index: int) -> float:
    return lib().rhzo_stateless_uniform(seed, stream, index)


# ----------------------------------------------------------------------------
# crates/ops/src/elementwise.rs
# ----------------------------------------------------------------------------

def sigmoid(x: float) -> float:
    return lib().rhzo_sigmoid(float(x))


def softplus(x: float) -> float:
    return lib().rhzo_softplus(float(x))


def l2norm(x, scale: float = 1.0) -> np.ndarray:
    x = _f64(x)
    out = np.empty_like(x)
    lib().rhzo_l2norm(x, x.size, float(scale), out)
    return out


# ----------------------------------------------------------------------------
# crates/ops/src/delta.rs
# ----------------------------------------------------------------------------

@dataclass
class DeltaInputs:
    """Per-position inputs for one head (delta.rs:13-29)."""

    head_dim: int
    q: np.ndarray
    k: np.ndarray
    v: np.ndarray
    alpha: np.ndarray
    beta: np.ndarray
    segment: np.ndarray = field(default=None)

    def __post_init__(self):
        self.q, self.k, self.v = _f64(self.q).ravel(), _f64(self.k).ravel(), _f64(self.v).ravel()
        self.alpha, self.beta = _f64(self.alpha).ravel(), _f64(self.beta).ravel()
        if self.segment is None:
            self.segment = np.zeros(len(self.alpha), dtype=np.int64)
        self.segment = np.ascontiguousarray(self.segment, dtype=np.int64).ravel()

    def __len__(self) -> int:  # delta.rs:34-36
        return len(self.alpha)

    def is_empty(self) -> bool:
        return len(self) == 0

    def is_consistent(self) -> bool:  # delta.rs:46-55
        return bool(lib().rhzo_inputs_consistent(self.head_dim, self.q.size, self.k.size,
                                                  self.v.size, self.alpha.size, self.beta.size,
                                                  self.segment.size))


@dataclass
class DeltaState:
    """d x d row-major state, S[i][j] at i*d + j (delta.rs:59-90)."""

    head_dim: int
    s: np.ndarray

    @staticmethod
    def zeros(d: int) -> "DeltaState":
        return DeltaState(d, np.zeros(d * d))

    def reset(self) -> None:
        self.s[:] = 0.0

    def max_abs_diff(self, other: "DeltaState") -> float:
        return float(np.max(np.abs(self.s - other.s), initial=0.0))

    def clone(self) -> "DeltaState":
        return DeltaState(self.head_dim, self.s.copy())


def gated_delta_step(state: DeltaState, q, k, v, alpha: float, beta: float) -> np.ndarray:
    """delta.rs:93-127; updates `state` in place and returns o_t."""
    d = state.head_dim
    o = np.empty(d)
    state.s = _f64(state.s)
    lib().rhzo_gated_delta_step(state.s, d, _f64(q), _f64(k), _f64(v), float(alpha),
                                float(beta), o)
    return o


def gated_delta_sequential(inp: DeltaInputs, init: DeltaState):
    """delta.rs:132-154 (resets at t = 0, so `init` is discarded)."""
    d, t = inp.head_dim, len(inp)
    out = np.empty(t * d)
    fin = np.empty(d * d)
    lib().rhzo_gated_delta_sequential(d, t, inp.q, inp.k, inp.v, inp.alpha, inp.beta,
                                      inp.segment, _f64(init.s), out, fin)
    return out, DeltaState(d, fin)


def gated_delta_scan_chunked(inp: DeltaInputs, init: DeltaState, chunk: int):
    """delta.rs:158-197."""
    d, t = inp.head_dim, len(inp)
    out = np.empty(t * d)
    fin = np.empty(d * d)
    lib().rhzo_gated_delta_scan_chunked(d, t, inp.q, inp.k, inp.v, inp.alpha, inp.beta,
                                        inp.segment, _f64(init.s), int(chunk), out, fin)
    return out, DeltaState(d, fin)


def gated_delta_multistep(inp: DeltaInputs, init: DeltaState, max_positions: int):
    """delta.rs:201-230; returns (outputs, [state after each position])."""
    d, t = inp.head_dim, len(inp)
    n = max(0, min(t, max_positions))
    outs = np.empty(max(n, 1) * d)
    states = np.empty(max(n, 1) * d * d)
    n = lib().rhzo_gated_delta_multistep(d, t, inp.q, inp.k, inp.v, inp.alpha, inp.beta,
                                         inp.segment, _f64(init.s), int(max_positions), outs,
                                         states)
    return outs[: n * d], [DeltaState(d, states[i * d * d:(i + 1) * d * d].copy())
                           for i in range(n)]


def gated_delta_step_loop(inp: DeltaInputs, init: DeltaState):
    """gated_delta_step over every position from `init`, no reset."""
    d, t = inp.head_dim, len(inp)
    out = np.empty(t * d)
    fin = np.empty(d * d)
    lib().rhzo_gated_delta_step_loop(d, t, inp.q, inp.k, inp.v, inp.alpha, inp.beta,
                                     _f64(init.s), out, fin)
    return out, DeltaState(d, fin)


def causal_conv1d_step(state: np.ndarray, weight, x: float, bias: float) -> float:
    """delta.rs:236-243; `state` (3 doubles) is updated in place."""
    assert state.dtype == np.float64 and state.flags.c_contiguous and state.size == 3
    return lib().rhzo_causal_conv1d_step(state, _f64(weight), float(x), float(bias))


# ----------------------------------------------------------------------------
# Batched drivers over the device layouts
# ----------------------------------------------------------------------------

def _threads(nthreads):
    return nthreads if nthreads else (os.cpu_count() or 1)


def gdr_varlen(cu_seqlens, q, k, v, alpha, beta, state_in=None, state_in_index=None,
               state_out_shape=None, state_out_index=None, nthreads=None):
    """Packed varlen step loop per (sequence, head).

    q/k/v: [tokens, H, d]; alpha/beta: [tokens, H]; state_in: [slots, H, d, d]
    indexed by state_in_index (default: sequence i -> i). Returns (o, state_out)
    where state_out has shape state_out_shape (default [n_seq, H, d, d]).
    """
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int64)
    q, k, v, alpha, beta = map(_f64, (q, k, v, alpha, beta))
    tokens, H, d = q.shape
    n_seq = cu.size - 1
    o = np.zeros_like(q)
    si = None if state_in is None else _f64(state_in)
    sii = None if state_in_index is None else np.ascontiguousarray(state_in_index, np.int64)
    soi = None if state_out_index is None else np.ascontiguousarray(state_out_index, np.int64)
    if soi is None:
        so = np.zeros((n_seq, H, d, d))
    elif si is not None and state_out_shape in (None, si.shape):
        so = si.copy()  # in-place slot pool: untouched slots keep their values
    else:
        so = np.zeros(state_out_shape)
    lib().rhzo_gdr_varlen(n_seq, cu, H, d, q, k, v, alpha, beta, _ptr(si), _ptr(sii), o,
                          _ptr(so), _ptr(soi), _threads(nthreads))
    return o, so


def gdr_dense(q, k, v, alpha, beta, state_in=None, nthreads=None):
    """Dense [B, T, H, d] batch; state_in [B, H, d, d] or None (zeros)."""
    q, k, v, alpha, beta = map(_f64, (q, k, v, alpha, beta))
    B, T, H, d = q.shape
    o = np.zeros_like(q)
    so = np.zeros((B, H, d, d))
    si = None if state_in is None else _f64(state_in)
    lib().rhzo_gdr_dense(B, T, H, d, q, k, v, alpha, beta, _ptr(si), o, _ptr(so),
                         _threads(nthreads))
    return o, so


def gdr_prep(cu_seqlens, xq, xk, xv, beta_logit, alpha_logit, a_head, conv_w, conv_b,
             conv_state=None, slots=None, zero_init=False, write_state=True, q_scale=1.0):
    """The Local block's input producer on the device layouts (gdr_oracle.c).

    xq/xk/xv: [tokens, H, d]; logits: [tokens, H]; a_head: [H];
    conv_w: [3, H, d, 4]; conv_b: [3, H, d]; conv_state: [slots, 3, H, d, 3]
    or None (zeros, nothing written). Returns (q, k, v, alpha, beta,
    conv_state_after)."""
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
    xq, xk, xv, bl, al, ah, w, b = map(_f64, (xq, xk, xv, beta_logit, alpha_logit, a_head,
                                             conv_w, conv_b))
    tokens, H, d = xq.shape
    n_seq = cu.size - 1
    q = np.zeros_like(xq); k = np.zeros_like(xq); v = np.zeros_like(xq)
    alpha = np.zeros((tokens, H)); beta = np.zeros_like(alpha)
    cs = None if conv_state is None else _f64(conv_state).copy()
    num_slots = 0 if cs is None else cs.shape[0]
    sl = None if slots is None else np.ascontiguousarray(slots, np.int32)
    lib().rhzo_gdr_prep(n_seq, cu, H, d, xq, xk, xv, bl, al, ah, w, b, _ptr(cs), _ptr(sl),
                        num_slots, int(zero_init), int(write_state), float(q_scale), q, k, v,
                        alpha, beta)
    return q, k, v, alpha, beta, cs


def groupnorm_heads(x, scale, eps: float):
    """norm.rs:48-60 on rows of [.., H, dh] values (x of any leading shape);
    each head uses scale[:dh]."""
    x = _f64(x)
    H, dh = x.shape[-2], x.shape[-1]
    rows = x.size // (H * dh)
    out = np.zeros_like(x)
    lib().rhzo_groupnorm_heads(x, rows, H, dh, _f64(scale), float(eps), out)
    return out


def gated_delta_backward(q, k, v, alpha, beta, d_o, segment=None, reset_at_start=True,
                         init=None, d_state_final=None):
    """Adjoint of the sequential recurrence for one head (gdr_oracle.c):
    q/k/v/d_o [T, d]; alpha/beta [T]; segment [T] int64 or None. Returns
    (dq, dk, dv, dalpha, dbeta, dinit)."""
    q, k, v, alpha, beta, d_o = map(_f64, (q, k, v, alpha, beta, d_o))
    T, d = q.shape
    dq, dk, dv = np.zeros_like(q), np.zeros_like(q), np.zeros_like(q)
    da, db = np.zeros(T), np.zeros(T)
    dinit = np.zeros((d, d))
    seg = None if segment is None else np.ascontiguousarray(segment, np.int64)
    ini = None if init is None else _f64(init)
    dsf = None if d_state_final is None else _f64(d_state_final)
    lib().rhzo_gated_delta_backward(d, T, q, k, v, alpha, beta, _ptr(seg), int(reset_at_start),
                                    _ptr(ini), d_o, _ptr(dsf), dq, dk, dv, da, db, _ptr(dinit))
    return dq, dk, dv, da, db, dinit


def make_qkv_gates(seed: int, tokens: int, H: int, d: int):
    """Seeded inputs with the benchmark distributions (see gdr_oracle.c)."""
    q = np.empty((tokens, H, d)); k = np.empty_like(q); v = np.empty_like(q)
    alpha = np.empty((tokens, H)); beta = np.empty_like(alpha)
    lib().rhzo_make_qkv_gates(seed, tokens, H, d, q, k, v, alpha, beta)
    return q, k, v, alpha, beta


def make_inputs(t: int, d: int, segments, seed: int) -> DeltaInputs:
    """The reference tests' fixture (delta.rs:254-280)."""
    q = np.empty(t * d); k = np.empty(t * d); v = np.empty(t * d)
    alpha = np.empty(t); beta = np.empty(t)
    lib().rhzo_make_test_inputs(t, d, seed, q, k, v, alpha, beta)
    return DeltaInputs(d, q, k, v, alpha, beta, np.asarray(segments, dtype=np.int64))


def make_normal(seed: int, stream: int, shape, sigma: float) -> np.ndarray:
    out = np.empty(shape)
    lib().rhzo_make_normal(seed, stream, out.size, sigma, out)
    return out
