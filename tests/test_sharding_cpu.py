"""Head sharding of the full layer on CPU process groups (gloo, 2 ranks):
the host-side layout logic of rhizome_b200.layer -- head ranges, the
rank-major all-gather, the unshard order -- against the unsharded f64 oracle.
The per-rank compute is the oracle here; on GPUs it is the chunked kernel."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rhizome_b200 import capi
from rhizome_b200.layer import gdr_layer_sharded, gdr_layer_sharded_slabs, head_range

B, T, H, D = 2, 70, 4, 8


def _problem():
    from oracle import oracle as O
    q, k, v, a, b = O.make_qkv_gates(11, B * T, H, D)
    sh = lambda x: x.reshape(B, T, *x.shape[1:])  # noqa: E731
    return tuple(sh(x) for x in (q, k, v, a, b))


def _oracle_compute(q, k, v, a, b):
    from oracle import oracle as O
    o, s = O.gdr_dense(q.numpy(), k.numpy(), v.numpy(), a.numpy(), b.numpy(), nthreads=1)
    return torch.from_numpy(o), torch.from_numpy(s)


def _torch_unshard(gathered):
    G, b, t, hs, d = gathered.shape
    return gathered.permute(1, 2, 0, 3, 4).reshape(b, t, G * hs, d)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = [torch.from_numpy(x) for x in _problem()]
        h0, h1 = head_range(H, world, rank)
        shard = [x[:, :, h0:h1].contiguous() for x in full]
        o, fin = gdr_layer_sharded(*shard, compute=_oracle_compute, unshard=_torch_unshard)
        ref_o, ref_s = _oracle_compute(*full)
        ok = torch.equal(o, ref_o) and torch.equal(fin, ref_s[:, h0:h1])
        q.put((rank, ok, (h0, h1)))
    finally:
        dist.destroy_process_group()


class _OracleSlabOps:
    """CPU stand-in for CudaSlabOps: torch packing and the f64 oracle's
    varlen scan, the state carried in f64 between slabs (the layer's f32
    pool receives a copy, as the device pool holds the kernels' f32 state)."""

    def __init__(self, b):
        self.B = b
        self.state = None

    def pack(self, x, t0, t1):
        return x[:, t0:t1].reshape(self.B * (t1 - t0), *x.shape[2:]).contiguous()

    def compute(self, q, k, v, a, b, pool, first, length):
        from oracle import oracle as O
        cu = np.arange(0, (self.B + 1) * length, length)
        o, self.state = O.gdr_varlen(cu, q.numpy(), k.numpy(), v.numpy(), a.numpy(), b.numpy(),
                                     state_in=None if first else self.state, nthreads=1)
        pool.copy_(torch.from_numpy(self.state))
        return torch.from_numpy(o)

    def unshard(self, gathered):
        G, tok, hs, d = gathered.shape
        return gathered.permute(1, 0, 2, 3).reshape(tok, G * hs, d)

    def unpack(self, out, slab, t0, t1):
        out[:, t0:t1] = slab.reshape(self.B, t1 - t0, *out.shape[2:])


def _slab_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = [torch.from_numpy(x) for x in _problem()]
        h0, h1 = head_range(H, world, rank)
        shard = [x[:, :, h0:h1].contiguous() for x in full]
        o, fin = gdr_layer_sharded_slabs(*shard, slab=64, slab_ops=_OracleSlabOps(B))
        ref_o, ref_s = _oracle_compute(*full)
        ok = torch.equal(o, ref_o) and torch.equal(fin, ref_s[:, h0:h1].float())
        q.put((rank, ok, (h0, h1)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_sharded_layer_matches_unsharded_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(results) == [(0, True, (0, 2)), (1, True, (2, 4))]


def test_slab_pipelined_layer_matches_unsharded_on_two_gloo_ranks():
    """The all-gather-overlapped form: T = 70 in slabs of 64 (a full slab
    and a ragged one), the state carried between them."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_slab_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(results) == [(0, True, (0, 2)), (1, True, (2, 4))]


def test_slab_must_be_a_multiple_of_64():
    x = torch.zeros(1, 64, 1, 8)
    a = torch.zeros(1, 64, 1)
    with pytest.raises(capi.InvalidArgument):
        gdr_layer_sharded_slabs(x, x, x, a, a, slab=100, slab_ops=_OracleSlabOps(1))


def test_head_range_rules():
    assert head_range(64, 8, 3) == (24, 32)
    assert head_range(16, 1, 0) == (0, 16)
    with pytest.raises(capi.ShapeError):
        head_range(10, 4, 0)
    with pytest.raises(capi.InvalidArgument):
        head_range(8, 2, 2)


def test_unshard_order_is_rank_major_heads():
    """gathered[r][.][.][hh] is head r * H/G + hh of the full layout."""
    G, Hs = 3, 2
    gathered = torch.arange(G * 1 * 2 * Hs * 1).reshape(G, 1, 2, Hs, 1)
    full = _torch_unshard(gathered)
    for r in range(G):
        for hh in range(Hs):
            assert torch.equal(full[:, :, r * Hs + hh], gathered[r, :, :, hh])
