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


class CudaSlabOps:
    """Device side of gdr_layer_sharded_slabs: slab rows packed by
    rhz_varlen_pack_tokens, the scan by rhz_gdr_varlen_fwd with the state
    carried in a [B, H/G, d, d] pool, outputs unsharded by rhz_heads_unshard
    and unpacked into the layer output by rhz_varlen_unpack_tokens."""

    def __init__(self, B: int, device):
        self.device = device
        self.B = B
        self._cu = {}
        self._ws = None  # the scan's scratch, shared by the slabs (one scan at a time)

    def rows(self, length: int) -> torch.Tensor:
        """cu_seqlens of a slab: batch row b holds packed rows [b L, (b+1) L)."""
        if length not in self._cu:
            self._cu[length] = torch.arange(0, (self.B + 1) * length, length, device=self.device,
                                            dtype=torch.int32)
        return self._cu[length]

    def pack(self, x: torch.Tensor, t0: int, t1: int) -> torch.Tensor:
        B, T = x.shape[0], x.shape[1]
        row = x[0, 0].numel() * x.element_size()
        out = torch.empty((B * (t1 - t0), *x.shape[2:]), device=x.device, dtype=x.dtype)
        capi.call("rhz_varlen_pack_tokens", out.data_ptr(), x.data_ptr() + t0 * row,
                  self.rows(t1 - t0).data_ptr(), B, T, row, ops._stream(x.device))
        return out

    def compute(self, q, k, v, a, b, pool, first: bool, length: int) -> torch.Tensor:
        o = torch.empty_like(q)
        H, d = q.shape[1], q.shape[2]
        flags = 1 if first else 0  # RHZ_FLAG_ZERO_INIT: the reset at t = 0
        need = ops.varlen_workspace_bytes(self.B, H, d, q.dtype)
        if need and (self._ws is None or self._ws.numel() < need):
            self._ws = torch.empty(need, device=q.device, dtype=torch.uint8)
        capi.call("rhz_gdr_varlen_fwd", o.data_ptr(), pool.data_ptr(), None,
                  self.rows(length).data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                  a.data_ptr(), b.data_ptr(), self.B, self.B * length, self.B, H, d,
                  ops._dt(q), flags, ops._p(self._ws) if need else None, need,
                  ops._stream(q.device))
        return o

    def unshard(self, gathered: torch.Tensor) -> torch.Tensor:
        G, tok, Hs, d = gathered.shape
        out = torch.empty((tok, G * Hs, d), device=gathered.device, dtype=gathered.dtype)
        capi.call("rhz_heads_unshard", out.data_ptr(), gathered.data_ptr(), G, tok, G * Hs, d,
                  gathered.element_size(), ops._stream(gathered.device))
        return out

    def unpack(self, out: torch.Tensor, slab: torch.Tensor, t0: int, t1: int) -> None:
        B, T = out.shape[0], out.shape[1]
        row = out[0, 0].numel() * out.element_size()
        capi.call("rhz_varlen_unpack_tokens", out.data_ptr() + t0 * row, slab.data_ptr(),
                  self.rows(t1 - t0).data_ptr(), B, T, row, ops._stream(out.device))


def gdr_layer_sharded_slabs(q, k, v, alpha, beta, slab: int = 4096, group=None,
                            slab_ops=None):
    """gdr_layer_sharded with the all-gather overlapped: T is cut into slabs
    (multiples of 64 positions, so the chunking and the result are those of
    the one-call layer, bitwise on the bf16 kernels), each rank scans slab j
    of its heads with the state carried from slab j-1, and slab j's outputs
    are all-gathered while slab j+1 computes. Returns (o [B, T, H, d] on
    every rank, this rank's final states [B, H/G, d, d]). `slab_ops` defaults
    to the CUDA kernels (CudaSlabOps); it is a parameter so the host-side
    orchestration can be checked against the f64 oracle on CPU process groups.
    """
    import torch.distributed as dist

    if slab <= 0 or slab % 64:
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"slab = {slab}: a positive multiple of 64")
    B, T, Hs, d = q.shape
    if slab_ops is None:
        # The CUDA slab moves address rows by raw pointer arithmetic: every
        # input must be a contiguous device tensor of this rank's [B, T, Hs]
        # shape (a head-slice view such as x[:, :, h0:h1] is not).
        ops._qkv(q, k, v, alpha, beta, (B, T))
    else:
        # Caller-supplied slab moves (the host-side check of the
        # orchestration) may use other dtypes; the shapes must still agree.
        for name, x in (("k", k), ("v", v)):
            if tuple(x.shape) != tuple(q.shape):
                raise capi.ShapeError(capi.RHZ_ERR_SHAPE, f"{name} must match q's shape")
        for name, x in (("alpha", alpha), ("beta", beta)):
            if tuple(x.shape) != (B, T, Hs):
                raise capi.ShapeError(capi.RHZ_ERR_SHAPE, f"{name} must be [{B}, {T}, {Hs}]")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    so = slab_ops or CudaSlabOps(B, q.device)
    out = torch.empty((B, T, world * Hs, d), device=q.device, dtype=q.dtype)
    pool = torch.zeros((B, Hs, d, d), device=q.device, dtype=torch.float32)
    pending = None  # (work, gathered, t0, t1) of the slab whose gather is in flight

    def finish(item):
        work, gathered, t0, t1 = item
        if work is not None:
            work.wait()
        so.unpack(out, so.unshard(gathered) if world > 1 else gathered[0], t0, t1)

    for t0 in range(0, T, slab):
        t1 = min(T, t0 + slab)
        parts = [so.pack(x, t0, t1) for x in (q, k, v, alpha, beta)]
        o_s = so.compute(*parts, pool, t0 == 0, t1 - t0)
        if world > 1:
            gathered = torch.empty((world, *o_s.shape), device=o_s.device, dtype=o_s.dtype)
            work = dist.all_gather_into_tensor(gathered.view(world * o_s.shape[0], *o_s.shape[1:]),
                                               o_s, group=group, async_op=True)
        else:
            gathered, work = o_s.unsqueeze(0), None
        if pending is not None:
            finish(pending)
        pending = (work, gathered, t0, t1)
    if pending is not None:
        finish(pending)
    return out, pool
