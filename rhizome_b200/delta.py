"""The reference's GDR API (crates/ops/src/delta.rs) on this backend.

Same names, argument meaning and results as the Rust functions: host f64
arrays in, host f64 arrays out, one head per call. The work runs on the GPU
through the C ABI -- the fp32 kernel (rtol 1e-5 against f64) by default, or
the bf16 tensor-core path with dtype="bf16". Inputs are checked like
DeltaInputs::is_consistent (delta.rs:46-55); an inconsistent input raises
capi.ShapeError (rhizome_core::Error::Shape) instead of panicking.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import capi, ops

_TORCH = {"f32": torch.float32, "bf16": torch.bfloat16}


@dataclass
class DeltaInputs:
    """Per-position inputs for one head (delta.rs:13-29): q, k, v are T x d
    row-major, alpha/beta/segment have T entries."""

    head_dim: int
    q: np.ndarray
    k: np.ndarray
    v: np.ndarray
    alpha: np.ndarray
    beta: np.ndarray
    segment: np.ndarray = field(default=None)

    def __post_init__(self):
        f = lambda x: np.ascontiguousarray(x, dtype=np.float64).ravel()  # noqa: E731
        self.q, self.k, self.v, self.alpha, self.beta = map(f, (self.q, self.k, self.v,
                                                                self.alpha, self.beta))
        if self.segment is None:
            self.segment = np.zeros(self.alpha.size, dtype=np.int64)
        self.segment = np.ascontiguousarray(self.segment, dtype=np.int64).ravel()

    def __len__(self) -> int:
        return self.alpha.size

    def is_empty(self) -> bool:
        return len(self) == 0

    def is_consistent(self) -> bool:
        t, d = len(self), self.head_dim
        return (d > 0 and self.q.size == t * d and self.k.size == t * d and self.v.size == t * d
                and self.beta.size == t and self.segment.size == t)


@dataclass
class DeltaState:
    """d x d state, S[i][j] at i * d + j (delta.rs:59-90)."""

    head_dim: int
    s: np.ndarray

    @staticmethod
    def zeros(d: int) -> "DeltaState":
        return DeltaState(d, np.zeros(d * d))

    def reset(self) -> None:
        self.s[:] = 0.0

    def max_abs_diff(self, other: "DeltaState") -> float:
        return float(np.max(np.abs(np.asarray(self.s) - np.asarray(other.s)), initial=0.0))

    def clone(self) -> "DeltaState":
        return DeltaState(self.head_dim, np.array(self.s, dtype=np.float64))


def _check(inp: DeltaInputs) -> None:
    if not inp.is_consistent():
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE,
                              f"inconsistent DeltaInputs: head_dim={inp.head_dim}, T={len(inp)}, "
                              f"|q|={inp.q.size}, |k|={inp.k.size}, |v|={inp.v.size}, "
                              f"|beta|={inp.beta.size}, |segment|={inp.segment.size}")


def _dev(x, dtype, device):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=dtype)


def _head_tensors(inp: DeltaInputs, dtype: str, device):
    t, d = len(inp), inp.head_dim
    td = _TORCH[dtype]
    q = _dev(inp.q.reshape(1, t, 1, d), td, device)
    k = _dev(inp.k.reshape(1, t, 1, d), td, device)
    v = _dev(inp.v.reshape(1, t, 1, d), td, device)
    a = _dev(inp.alpha.reshape(1, t, 1), torch.float32, device)
    b = _dev(inp.beta.reshape(1, t, 1), torch.float32, device)
    seg = _dev(inp.segment.reshape(1, t), torch.int64, device)
    return q, k, v, a, b, seg


def gated_delta_step(state: DeltaState, q, k, v, alpha: float, beta: float, *, dtype="f32",
                     device="cuda") -> np.ndarray:
    """delta.rs:93-127: updates `state` in place and returns o_t."""
    d = state.head_dim
    q, k, v = (np.asarray(x, dtype=np.float64).ravel() for x in (q, k, v))
    if d <= 0 or q.size != d or k.size != d or v.size != d or np.asarray(state.s).size != d * d:
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE, "gated_delta_step: vector/state sizes do not match head_dim")
    td = _TORCH[dtype]
    pool = _dev(np.asarray(state.s).reshape(1, 1, d, d), torch.float32, device)
    o = ops.gdr_step(_dev(q.reshape(1, 1, d), td, device), _dev(k.reshape(1, 1, d), td, device),
                     _dev(v.reshape(1, 1, d), td, device),
                     torch.full((1, 1), float(alpha), device=device, dtype=torch.float32),
                     torch.full((1, 1), float(beta), device=device, dtype=torch.float32), pool)
    state.s = pool.double().cpu().numpy().ravel()
    return o.double().cpu().numpy().ravel()


def gated_delta_sequential(inp: DeltaInputs, init: DeltaState, *, dtype="f32", device="cuda"):
    """delta.rs:132-154. Returns (outputs T*d, final DeltaState); `init` is
    discarded by the reset at t = 0, as in the reference."""
    return _scan(inp, init, None, dtype, device)


def gated_delta_scan_chunked(inp: DeltaInputs, init: DeltaState, chunk: int, *, dtype="f32",
                             device="cuda"):
    """delta.rs:158-197; same result as gated_delta_sequential."""
    return _scan(inp, init, chunk, dtype, device)


def _scan(inp, init, chunk, dtype, device):
    _check(inp)
    d, t = inp.head_dim, len(inp)
    if t == 0:
        return np.zeros(0), init.clone()  # the loop never runs: init.clone()
    q, k, v, a, b, seg = _head_tensors(inp, dtype, device)
    seg_arg = seg if np.any(inp.segment != inp.segment[0]) else None
    if chunk is None:
        o, fin = ops.gdr_sequential(q, k, v, a, b, segment=seg_arg)
    else:
        o, fin = ops.gdr_scan_chunked(q, k, v, a, b, chunk=int(chunk), segment=seg_arg)
    return (o.double().cpu().numpy().ravel(),
            DeltaState(d, fin.double().cpu().numpy().ravel()))


def gated_delta_multistep(inp: DeltaInputs, init: DeltaState, max_positions: int, *,
                          dtype="f32", device="cuda"):
    """delta.rs:201-230: at most max_positions steps; returns (outputs,
    [state after each position]). Resets at t = 0 (so `init` is discarded,
    as in the reference) and at segment changes."""
    _check(inp)
    d, t = inp.head_dim, len(inp)
    n = max(0, min(t, int(max_positions)))
    if n == 0:
        return np.zeros(0), []
    q, k, v, a, b, seg = _head_tensors(inp, dtype, device)
    outs, states = ops.gdr_multistep(q, k, v, a, b, max_positions=n, segment=seg)
    outs = outs.double().cpu().numpy().reshape(n * d)
    st = states.double().cpu().numpy().reshape(n, d * d)
    return outs, [DeltaState(d, st[i].copy()) for i in range(n)]
