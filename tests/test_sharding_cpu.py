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
from rhizome_b200.layer import gdr_layer_sharded, head_range

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
