"""Chunked (WY form) forward and backward of the gated delta rule in f64
numpy -- test infrastructure, the restatement a chunked tensor-core backward
is checked against.

Per chunk of C positions from state S0 (the forward the chunked kernels
run, gdr_chunk_tc.cu): P[t][s] = prod alpha over (s, t], gamma_t = P[t][-1],
A = diag(beta) (P . K K^T) strictly lower, T = (I + A)^-1, U = T diag(beta) V,
W = T diag(beta gamma) K, Delta = U - W S0^T,
O = diag(gamma) Q S0^T + (P . Q K^T) Delta,
S_C = gamma_{C-1} S0 + Delta^T diag(P[C-1]) K.
chunk_bwd differentiates those products in reverse (every step a matrix
product or an elementwise mask), and chunked_backward chains the chunks
backwards through dS0. The reference has no backward code; tests pin this
against the sequential adjoint in gdr_oracle.c (itself pinned to central
differences). Positive alphas only (the log-decay form divides by alpha).
"""
import numpy as np


def chunk_fwd(q, k, v, a, b, S0):
    C = q.shape[0]
    gl = np.cumsum(np.log(a))
    g = np.exp(gl)
    P = np.tril(np.exp(gl[:, None] - gl[None, :]))
    KK, QK = k @ k.T, q @ k.T
    A = np.tril(b[:, None] * P * KK, -1)
    T = np.linalg.inv(np.eye(C) + A)
    Y = b[:, None] * v
    Z = (b * g)[:, None] * k
    U, W = T @ Y, T @ Z
    D = U - W @ S0.T
    M = P * QK
    O_ = g[:, None] * (q @ S0.T) + M @ D
    pL = P[C - 1]
    SC = g[C - 1] * S0 + D.T @ (pL[:, None] * k)
    return O_, SC, dict(gl=gl, g=g, P=P, KK=KK, QK=QK, T=T, Y=Y, Z=Z, D=D, M=M, pL=pL)


def chunk_bwd(q, k, v, a, b, S0, dO, dSC):
    C = q.shape[0]
    _, _, c = chunk_fwd(q, k, v, a, b, S0)
    g, P, KK, QK, T, Y, Z, D, M, pL = (c[x] for x in ('g', 'P', 'KK', 'QK', 'T', 'Y', 'Z', 'D', 'M', 'pL'))
    dD = M.T @ dO + (pL[:, None] * k) @ dSC.T
    dM = np.tril(dO @ D.T)
    dS0 = dO.T @ (g[:, None] * q) + g[C - 1] * dSC - dD.T @ (T @ Z)
    dq = g[:, None] * (dO @ S0) + (dM * P) @ k
    dk = (dM * P).T @ q
    dP = dM * QK
    dg = np.sum(dO * (q @ S0.T), axis=1)
    dg[C - 1] += np.sum(dSC * S0)
    DdS = D @ dSC
    dk += pL[:, None] * DdS
    dP[C - 1] += np.sum(k * DdS, axis=1)
    dU, dW = dD, -dD @ S0
    dY, dT = T.T @ dU, dU @ Y.T
    dZ = T.T @ dW
    dT += dW @ Z.T
    dv = b[:, None] * dY
    db = np.sum(dY * v, axis=1)
    dk += (b * g)[:, None] * dZ
    dbg = np.sum(dZ * k, axis=1)
    db += dbg * g
    dg += dbg * b
    dA = np.tril(-T.T @ dT @ T.T, -1)
    db += np.sum(dA * P * KK, axis=1)
    dP += dA * b[:, None] * KK
    dKK = dA * b[:, None] * P
    dk += dKK @ k + dKK.T @ k
    PP = np.tril(dP * P)
    dgl = PP.sum(axis=1) - PP.sum(axis=0) + dg * g
    dloga = np.cumsum(dgl[::-1])[::-1]
    da = dloga / a
    return dq, dk, dv, da, db, dS0


def chunked_backward(q, k, v, a, b, dO, C, dSf=None):
    T_, d = q.shape
    n = (T_ + C - 1) // C
    S = [np.zeros((d, d))]
    for c in range(n):
        sl = slice(c * C, min(T_, (c + 1) * C))
        _, SC, _ = chunk_fwd(q[sl], k[sl], v[sl], a[sl], b[sl], S[-1])
        S.append(SC)
    dq, dk, dv = np.zeros_like(q), np.zeros_like(q), np.zeros_like(q)
    da, db = np.zeros(T_), np.zeros(T_)
    dS = np.zeros((d, d)) if dSf is None else dSf
    for c in reversed(range(n)):
        sl = slice(c * C, min(T_, (c + 1) * C))
        r = chunk_bwd(q[sl], k[sl], v[sl], a[sl], b[sl], S[c], dO[sl], dS)
        dq[sl], dk[sl], dv[sl], da[sl], db[sl], dS = r
    return dq, dk, dv, da, db
