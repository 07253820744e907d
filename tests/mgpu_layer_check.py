"""Run under torchrun with 2+ GPUs (launched by tests/test_gpu_layer.py):
the head-sharded layer over NCCL equals the single-GPU full layer, bitwise."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from rhizome_b200 import ops  # noqa: E402
from rhizome_b200.layer import gdr_layer_sharded, gdr_layer_sharded_slabs, head_range  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    B, T, H, D = 2, 300, 8, 128
    g = torch.Generator(device="cuda").manual_seed(42)
    n = torch.nn.functional.normalize
    q = n(torch.randn(B, T, H, D, device="cuda", generator=g), dim=-1).bfloat16()
    k = n(torch.randn(B, T, H, D, device="cuda", generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16()
    b = torch.sigmoid(torch.randn(B, T, H, device="cuda", generator=g))
    a = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, device="cuda", generator=g) + 2))
    h0, h1 = head_range(H, world, rank)
    sh = [x[:, :, h0:h1].contiguous() for x in (q, k, v, a, b)]
    o, fin = gdr_layer_sharded(*sh)
    ref_o, ref_s = ops.gdr_scan_chunked(q, k, v, a, b)
    torch.cuda.synchronize()
    ok = torch.equal(o, ref_o) and torch.equal(fin, ref_s[:, h0:h1])
    # the all-gather-overlapped form, three slabs (128, 128, 44 positions)
    o2, fin2 = gdr_layer_sharded_slabs(*sh, slab=128)
    torch.cuda.synchronize()
    ok = ok and torch.equal(o2, ref_o) and torch.equal(fin2, ref_s[:, h0:h1])
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        print("MGPU_LAYER_OK" if flag.item() == 0 else "MGPU_LAYER_MISMATCH", flush=True)
    return 0 if flag.item() == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
