"""The no-allocation entry point, rhz_varlen_segments_to_cu_seqlens_noalloc.

It exists for callers that cannot allocate device memory -- a plan executor
that owns only the arena its planner sized in advance, or a serving process
that reserved all device memory for its state slots -- so its scan scratch
is a fixed 64 KiB array inside the library instead of a caller workspace.
These tests call it through the C ABI and compare it with the workspace
entry point, bit for bit (it is index work), on two calls in a row with
different inputs, so a stale value left in the shared array by the first call
would show up in the second. This file sorts last so a run that stops at the
first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

from rhizome_b200 import capi, ops

pytestmark = pytest.mark.gpu


def _noalloc(seg: torch.Tensor):
    B, T = seg.shape
    cu = torch.full((B * T + 1,), -7, device=seg.device, dtype=torch.int32)
    n = torch.full((1,), -7, device=seg.device, dtype=torch.int32)
    stream = torch.cuda.current_stream(seg.device).cuda_stream
    st = capi.lib().rhz_varlen_segments_to_cu_seqlens_noalloc(
        cu.data_ptr(), n.data_ptr(), seg.data_ptr(), B, T, stream)
    capi.check(st)
    return cu, n


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    # Second call has more tiles than the first and different boundaries.
    for call, (B, T, p) in enumerate([(3, 5000, 0.01), (2, 40_000, 0.2)]):
        rng = np.random.default_rng(100 + call)
        seg = np.cumsum(rng.random((B, T)) < p, axis=1).astype(np.int64)
        dseg = torch.from_numpy(seg).cuda()
        ref_cu, ref_n = ops.segments_to_cu_seqlens(dseg)
        cu, n = _noalloc(dseg)
        torch.cuda.synchronize()
        n_ref = int(ref_n.item())
        assert int(n.item()) == n_ref, f"call {call}"
        assert torch.equal(cu[: n_ref + 1], ref_cu[: n_ref + 1]), f"call {call}"


def test_noalloc_rejects_sizes_beyond_its_limit():
    lim = capi.RHZ_NOALLOC_MAX_POSITIONS
    seg = torch.zeros(8, device="cuda", dtype=torch.int64)
    st = capi.lib().rhz_varlen_segments_to_cu_seqlens_noalloc(
        seg.data_ptr(), seg.data_ptr(), seg.data_ptr(), 2, lim // 2 + 1, None)
    assert st == capi.RHZ_ERR_SHAPE
    assert b"no-allocation limit" in capi.lib().rhz_last_error()
