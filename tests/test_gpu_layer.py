"""Head sharding of the full layer on GPUs: the unshard/shard moves are
bit-exact, per-shard computes reassemble the unsharded layer bitwise, and
(with 2+ GPUs) the NCCL all-gather path equals the single-GPU layer."""
import os
import socket
import subprocess
import sys

import pytest
import torch

from rhizome_b200 import ops
from rhizome_b200.layer import gdr_layer_sharded_slabs, head_range, heads_shard, heads_unshard

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("G", [1, 2, 8])
def test_unshard_and_shard_are_exact_inverses(dtype, G):
    B, T, H, D = 2, 33, 16, 128
    full = torch.randn(B, T, H, D, device="cuda").to(dtype)
    gathered = heads_shard(full, G)
    ref = full.view(B, T, G, H // G, D).permute(2, 0, 1, 3, 4)
    assert torch.equal(gathered, ref)
    assert torch.equal(heads_unshard(gathered), full)


def test_sharded_computes_reassemble_the_full_layer_bitwise():
    B, T, H, D, G = 2, 200, 8, 128, 4
    g = torch.Generator(device="cuda").manual_seed(3)
    n = torch.nn.functional.normalize
    q = n(torch.randn(B, T, H, D, device="cuda", generator=g), dim=-1).bfloat16()
    k = n(torch.randn(B, T, H, D, device="cuda", generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16()
    b = torch.sigmoid(torch.randn(B, T, H, device="cuda", generator=g))
    a = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, device="cuda", generator=g) + 2))
    ref_o, ref_s = ops.gdr_scan_chunked(q, k, v, a, b)
    outs = []
    for r in range(G):
        h0, h1 = head_range(H, G, r)
        o, s = ops.gdr_scan_chunked(*(x[:, :, h0:h1].contiguous() for x in (q, k, v, a, b)))
        assert torch.equal(s, ref_s[:, h0:h1])
        outs.append(o)
    assert torch.equal(heads_unshard(torch.stack(outs)), ref_o)


@pytest.mark.parametrize("T,slab", [(300, 128), (64, 64), (130, 4096)])
def test_slab_pipelined_layer_one_gpu_is_bitwise_the_one_call_layer(T, slab):
    """Slabs of 64-multiples with the state carried in fp32 between them give
    the one-call chunked result bit for bit (one rank: no all-gather)."""
    B, H, D = 2, 4, 128
    g = torch.Generator(device="cuda").manual_seed(T)
    n = torch.nn.functional.normalize
    q = n(torch.randn(B, T, H, D, device="cuda", generator=g), dim=-1).bfloat16()
    k = n(torch.randn(B, T, H, D, device="cuda", generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16()
    b = torch.sigmoid(torch.randn(B, T, H, device="cuda", generator=g))
    a = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, device="cuda", generator=g) + 2))
    o, fin = gdr_layer_sharded_slabs(q, k, v, a, b, slab=slab)
    ref_o, ref_s = ops.gdr_scan_chunked(q, k, v, a, b)
    torch.cuda.synchronize()
    assert torch.equal(o, ref_o) and torch.equal(fin, ref_s)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_sharded_layer_on_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", os.path.join(ROOT, "tests", "mgpu_layer_check.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert res.returncode == 0 and "MGPU_LAYER_OK" in res.stdout, res.stdout[-2000:] + res.stderr[-2000:]
