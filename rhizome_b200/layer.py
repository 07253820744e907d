"""The full Local-block GDR layer with its heads split over GPUs.

The recurrence never mixes heads (crates/ops/src/delta.rs:93-127 is one head
at a time), so H heads split evenly over G ranks need no state exchange:
rank r runs the chunked kernel on heads [r H/G, (r+1) H/G) of every sequence
and the only collective is an all-gather of the per-head outputs. NCCL
gathers the ranks' [B, T, H/G, d] outputs rank-major; rhz_heads_unshard puts
them back in [B, T, H, d] order (i.e. [B, T, H*d]).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import capi, ops


def head_range(H: int, world: int, rank: int) -> tuple[int, int]:
    """Heads owned by `rank`: an even split of H over `world` ranks."""
    if world < 1 or not 0 <= rank < world:
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"rank {rank} of world {world}")
    if H % world:
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE, f"H = {H} heads do not split evenly over {world} ranks")
    hs = H // world
    return rank * hs, (rank + 1) * hs


def heads_unshard(gathered: torch.Tensor) -> torch.Tensor:
    """[G, B, T, H/G, d] (rank-major all-gather result) -> [B, T, H, d]."""
    G, B, T, Hs, d = gathered.shape
    out = torch.empty((B, T, G * Hs, d), device=gathered.device, dtype=gathered.dtype)
    capi.call("rhz_heads_unshard", out.data_ptr(), gathered.data_ptr(), G, B * T, G * Hs, d,
              gathered.element_size(), torch.cuda.current_stream(gathered.device).cuda_stream)
    return out


def heads_shard(full: torch.Tensor, G: int) -> torch.Tensor:
    """[B, T, H, d] -> [G, B, T, H/G, d] (the inverse of heads_unshard)."""
    B, T, H, d = full.shape
    if H % G:
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE, f"H = {H} heads do not split evenly over {G} ranks")
    out = torch.empty((G, B, T, H // G, d), device=full.device, dtype=full.dtype)
    capi.call("rhz_heads_shard", out.data_ptr(), full.data_ptr(), G, B * T, H, d,
              full.element_size(), torch.cuda.current_stream(full.device).cuda_stream)
    return out


def gdr_layer_sharded(q, k, v, alpha, beta, group=None, chunk: int = 64,
                      compute: Optional[Callable] = None,
                      unshard: Optional[Callable] = None):
    """One rank's part of the head-sharded layer.

    q, k, v: this rank's heads, [B, T, H/G, d]; alpha, beta: [B, T, H/G].
    Returns (o [B, T, H, d] on every rank, this rank's final states
    [B, H/G, d, d]). `compute` and `unshard` default to the CUDA kernels
    (gdr_scan_chunked and rhz_heads_unshard); they are parameters only so the
    host-side layout logic can be exercised against the f64 oracle on CPU
    process groups.
    """
    import torch.distributed as dist

    compute = compute or (lambda *a: ops.gdr_scan_chunked(*a, chunk=chunk))
    unshard = unshard or heads_unshard
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    o_shard, fin = compute(q, k, v, alpha, beta)
    if world == 1:
        return o_shard, fin
    o_shard = o_shard.contiguous()
    # Rank-major gather buffer, concatenated along dim 0 (the form every
    # backend accepts), viewed as [G, B, T, H/G, d].
    gathered = torch.empty((world * o_shard.shape[0], *o_shard.shape[1:]), device=o_shard.device,
                           dtype=o_shard.dtype)
    dist.all_gather_into_tensor(gathered, o_shard, group=group)
    return unshard(gathered.view(world, *o_shard.shape)), fin
