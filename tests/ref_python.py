"""A second, independent transcription of crates/ops/src/delta.rs:93-197 in
pure Python floats (IEEE f64, no contraction -- the same rounding as Rust's
f64). Small cases only; used to check the C oracle bit for bit."""


def step(s, d, q, k, v, alpha, beta):
    """gated_delta_step, delta.rs:93-127 (s is a flat list, updated in place)."""
    sk = [0.0] * d
    for i in range(d):
        acc = 0.0
        for j in range(d):
            acc += s[i * d + j] * k[j]
        sk[i] = acc
    for i in range(d):
        for j in range(d):
            decayed = alpha * (s[i * d + j] - beta * sk[i] * k[j])
            s[i * d + j] = decayed + beta * v[i] * k[j]
    o = [0.0] * d
    for i in range(d):
        acc = 0.0
        for j in range(d):
            acc += s[i * d + j] * q[j]
        o[i] = acc
    return o


def sequential(d, q, k, v, alpha, beta, segment, init):
    """gated_delta_sequential, delta.rs:132-154."""
    s = list(init)
    out = []
    prev = None
    for t in range(len(alpha)):
        if prev != segment[t]:
            s = [0.0] * (d * d)
            prev = segment[t]
        out.extend(step(s, d, q[t * d:(t + 1) * d], k[t * d:(t + 1) * d],
                        v[t * d:(t + 1) * d], alpha[t], beta[t]))
    return out, s
