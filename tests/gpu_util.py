"""Shared helpers for the GPU parity tests: seeded inputs from the oracle's
Philox generator, rounded to exactly what the device kernels receive."""
from __future__ import annotations

import contextlib

import numpy as np
import torch

from oracle import oracle as O
from rhizome_b200 import ops
from tests.tolerance import bf16_round


def to_dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def host(x: torch.Tensor) -> np.ndarray:
    return x.double().cpu().numpy()


def make_inputs(seed: int, tokens: int, H: int, d: int, dtype: str):
    """q, k, v [tokens, H, d], alpha, beta [tokens, H] as f64 host arrays whose
    values are exactly representable in the kernel's dtype (bf16 for q/k/v in
    the bf16 path; f32 otherwise)."""
    q, k, v, a, b = O.make_qkv_gates(seed, tokens, H, d)
    rnd = bf16_round if dtype == "bf16" else (lambda x: x.astype(np.float32).astype(np.float64))
    q, k, v = rnd(q), rnd(k), rnd(v)
    a = a.astype(np.float32).astype(np.float64)
    b = b.astype(np.float32).astype(np.float64)
    return q, k, v, a, b


TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16}


def device_inputs(q, k, v, a, b, dtype: str):
    td = TORCH_DT[dtype]
    return (to_dev(q, td), to_dev(k, td), to_dev(v, td), to_dev(a, torch.float32),
            to_dev(b, torch.float32))


@contextlib.contextmanager
def chunk_form(name: str):
    """Pin the tensor-core chunked scan to one form ("pair", "solo", "auto")
    for the duration of the block."""
    prev = ops.set_chunk_kernel(name)
    try:
        yield
    finally:
        ops.set_chunk_kernel(prev)
