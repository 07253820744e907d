"""torch-facing wrappers of the C ABI (device tensors in, device tensors out).

torch only supplies device memory and the current stream; every op is one
C-ABI call into librhizome_gdr.so. Layouts follow include/rhizome_gdr.h:
q/k/v/o [tokens, H, d] (dense batches [B, T, H, d]), alpha/beta [tokens, H]
f32, states [n, H, d, d] f32 with S[i][j], i the v index and j the k index.
"""
from __future__ import annotations

import ctypes

import torch

from . import capi

_DTYPES = {torch.float32: capi.RHZ_DTYPE_F32, torch.bfloat16: capi.RHZ_DTYPE_BF16}


def _dt(x: torch.Tensor) -> int:
    try:
        return _DTYPES[x.dtype]
    except KeyError:
        raise capi.DtypeError(capi.RHZ_ERR_DTYPE, f"unsupported dtype {x.dtype}") from None


def _p(x):
    return None if x is None else x.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _need(x: torch.Tensor, name: str, dtype=None, shape=None):
    # Shape and dtype first (the most specific message), then layout and device.
    if shape is not None and tuple(x.shape) != tuple(shape):
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE, f"{name} has shape {tuple(x.shape)}, expected {tuple(shape)}")
    if dtype is not None and x.dtype != dtype:
        raise capi.DtypeError(capi.RHZ_ERR_DTYPE, f"{name} must be {dtype}, got {x.dtype}")
    if not x.is_contiguous():
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"{name} must be contiguous")
    if not x.is_cuda:
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"{name} must be a CUDA tensor")


def _pool(state_pool, name, H, d):
    """A state pool [slots, H, d, d] f32; returns its slot count."""
    if state_pool.dim() != 4 or tuple(state_pool.shape[1:]) != (H, d, d):
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE,
                              f"{name} shape {tuple(state_pool.shape)} != [slots, {H}, {d}, {d}]")
    _need(state_pool, name, torch.float32)
    return state_pool.shape[0]


def _workspace(ws, nbytes, dev):
    """The caller's workspace (or a new one of nbytes) and its real size in bytes."""
    if ws is None:
        ws = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    _need(ws, "workspace")
    if ws.device != dev:
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"workspace is on {ws.device}, q on {dev}")
    return ws, ws.numel() * ws.element_size()


def _qkv(q, k, v, alpha, beta, lead):
    d = q.shape[-1]
    H = q.shape[-2]
    for name, x in (("q", q), ("k", k), ("v", v)):
        _need(x, name, q.dtype, (*lead, H, d))
    _need(alpha, "alpha", torch.float32, (*lead, H))
    _need(beta, "beta", torch.float32, (*lead, H))
    return H, d


def gdr_step(q, k, v, alpha, beta, state_pool, slot_idx=None, out=None):
    """gated_delta_step (delta.rs:93-127) for n sequences x H heads, in place
    on state_pool[slot_idx[i]]. q/k/v [n, H, d]; returns o [n, H, d]."""
    n = q.shape[0]
    H, d = _qkv(q, k, v, alpha, beta, (n,))
    if out is not None:
        _need(out, "out", q.dtype, tuple(q.shape))
    _pool(state_pool, "state_pool", H, d)
    if slot_idx is not None:
        _need(slot_idx, "slot_idx", torch.int32, (n,))
    o = torch.empty_like(q) if out is None else out
    capi.call("rhz_gdr_step", _p(o), _p(state_pool), _p(slot_idx), _p(q), _p(k), _p(v),
              _p(alpha), _p(beta), n, state_pool.shape[0], H, d, _dt(q), _stream(q.device))
    return o


def gdr_multistep(q, k, v, alpha, beta, max_positions=8, segment=None, state_pool=None,
                  slot_idx=None):
    """gated_delta_multistep (delta.rs:201-230) for n sequences: q/k/v
    [n, T, H, d]. Returns (outs [n, Tn, H, d], states [n, Tn, H, d, d]) with
    Tn = min(T, max_positions). Without a state_pool the state starts at zero
    and resets at segment changes (the reference); with one, sequence i starts
    from state_pool[slot_idx[i]] and the pool is left unchanged."""
    n, T = q.shape[0], q.shape[1]
    H, d = _qkv(q, k, v, alpha, beta, (n, T))
    Tn = max(0, min(T, int(max_positions)))
    if segment is not None:
        _need(segment, "segment", torch.int64, (n, T))
    num_slots = 0 if state_pool is None else _pool(state_pool, "state_pool", H, d)
    if slot_idx is not None:
        _need(slot_idx, "slot_idx", torch.int32, (n,))
    outs = torch.empty((n, Tn, H, d), device=q.device, dtype=q.dtype)
    states = torch.empty((n, Tn, H, d, d), device=q.device, dtype=torch.float32)
    capi.call("rhz_gdr_multistep", _p(outs), _p(states), _p(state_pool), _p(slot_idx), _p(q),
              _p(k), _p(v), _p(alpha), _p(beta), _p(segment), n, T, int(max_positions), num_slots,
              H, d, _dt(q), _stream(q.device))
    return outs, states


def gdr_prep(xq, xk, xv, beta_logit, alpha_logit, a_head, conv_w, conv_b, conv_state=None,
             slot_idx=None, cu_seqlens=None, q_scale=1.0, zero_init=False, write_state=True):
    """The Local block's input producer: causal depthwise conv of kernel 4
    (delta.rs:236-243) carried per sequence in conv_state slots, then
    q = l2norm(conv q) * q_scale, k = l2norm(conv k), v = conv v,
    beta = sigmoid(beta_logit), alpha = exp(-softplus(a_head) softplus(alpha_logit)).

    Dense: xq/xk/xv [B, T, H, d] (cu_seqlens None, one sequence per batch
    row); packed: [tokens, H, d] with cu_seqlens [n_seq + 1] int32. Logits
    [.., H] f32; a_head [H]; conv_w [3, H, d, 4]; conv_b [3, H, d];
    conv_state [slots, 3, H, d, 3] f32 (updated in place unless
    write_state is False). Returns (q, k, v, alpha, beta)."""
    H, d = xq.shape[-2], xq.shape[-1]
    for t, name in ((xk, "xk"), (xv, "xv")):
        _need(t, name, xq.dtype, tuple(xq.shape))
    if cu_seqlens is None:
        B, T = xq.shape[0], xq.shape[1]
        n_seq, seq_len, total = B, T, B * T
    else:
        _need(cu_seqlens, "cu_seqlens", torch.int32)
        n_seq, seq_len, total = cu_seqlens.numel() - 1, 0, xq.shape[0]
    for t, name in ((beta_logit, "beta_logit"), (alpha_logit, "alpha_logit")):
        _need(t, name, torch.float32, tuple(xq.shape[:-1]))
    _need(a_head, "a_head", torch.float32, (H,))
    _need(conv_w, "conv_w", torch.float32, (3, H, d, 4))
    _need(conv_b, "conv_b", torch.float32, (3, H, d))
    num_slots = 0
    if conv_state is not None:
        _need(conv_state, "conv_state", torch.float32)
        num_slots = conv_state.shape[0]
    if slot_idx is not None:
        _need(slot_idx, "slot_idx", torch.int32, (n_seq,))
    q, k, v = torch.empty_like(xq), torch.empty_like(xq), torch.empty_like(xq)
    alpha = torch.empty(xq.shape[:-1], device=xq.device, dtype=torch.float32)
    beta = torch.empty_like(alpha)
    flags = (capi.RHZ_FLAG_ZERO_INIT if zero_init else 0) | \
            (0 if write_state else capi.RHZ_FLAG_NO_STATE_WRITE)
    capi.call("rhz_gdr_prep", _p(q), _p(k), _p(v), _p(alpha), _p(beta), _p(xq), _p(xk), _p(xv),
              _p(beta_logit), _p(alpha_logit), _p(a_head), _p(conv_w), _p(conv_b), _p(conv_state),
              _p(slot_idx), _p(cu_seqlens), n_seq, seq_len, total, num_slots, H, d,
              float(q_scale), _dt(xq), flags, _stream(xq.device))
    return q, k, v, alpha, beta


def workspace_bytes(B: int, T: int, H: int = 1, d: int = 1, dtype: torch.dtype = torch.float32,
                    has_segment: bool = True) -> int:
    """Scratch of gdr_sequential / gdr_scan_chunked (see rhz_gdr_workspace_bytes)."""
    return int(capi.lib().rhz_gdr_workspace_bytes(B, T, H, d, _DTYPES.get(dtype, -1),
                                                  1 if has_segment else 0))


def varlen_workspace_bytes(n_seq: int, H: int, d: int, dtype: torch.dtype) -> int:
    """Scratch of gdr_varlen_fwd(_norm) for n_seq sequences."""
    return int(capi.lib().rhz_gdr_varlen_workspace_bytes(n_seq, H, d, _DTYPES.get(dtype, -1)))


def _seq_common(name, q, k, v, alpha, beta, segment, state_init, chunk, with_state, workspace):
    B, T = q.shape[0], q.shape[1]
    H, d = _qkv(q, k, v, alpha, beta, (B, T))
    if segment is not None:
        _need(segment, "segment", torch.int64, (B, T))
    if state_init is not None:
        _need(state_init, "state_init", torch.float32, (B, H, d, d))
    o = torch.empty_like(q)
    fin = torch.empty((B, H, d, d), device=q.device, dtype=torch.float32) if with_state else None
    ws, nbytes = None, 0
    need = workspace_bytes(B, T, H, d, q.dtype, segment is not None)
    if need > 0 or workspace is not None:
        ws, nbytes = _workspace(workspace, need, q.device)
    args = [_p(o), _p(fin), _p(q), _p(k), _p(v), _p(alpha), _p(beta), _p(segment), _p(state_init)]
    if name == "rhz_gdr_scan_chunked":
        args.append(chunk)
    args += [B, T, H, d, _dt(q), _p(ws), nbytes, _stream(q.device)]
    capi.call(name, *args)
    return o, fin


def gdr_sequential(q, k, v, alpha, beta, segment=None, state_init=None, with_state=True,
                   workspace=None):
    """gated_delta_sequential (delta.rs:132-154) on [B, T, H, d]: resets at
    t = 0 and at segment changes; state_init is accepted and, as in the
    reference, never reaches the result. Returns (o, final_state|None)."""
    return _seq_common("rhz_gdr_sequential", q, k, v, alpha, beta, segment, state_init, 0,
                       with_state, workspace)


def gdr_scan_chunked(q, k, v, alpha, beta, chunk=64, segment=None, state_init=None,
                     with_state=True, workspace=None):
    """gated_delta_scan_chunked (delta.rs:158-197); the result does not
    depend on `chunk`."""
    return _seq_common("rhz_gdr_scan_chunked", q, k, v, alpha, beta, segment, state_init, chunk,
                       with_state, workspace)


def _need_host(x: torch.Tensor, name: str, dtype=None, shape=None):
    if x.is_cuda:
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"{name} must be a host (CPU) tensor")
    if not x.is_contiguous():
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"{name} must be contiguous")
    if dtype is not None and x.dtype != dtype:
        raise capi.DtypeError(capi.RHZ_ERR_DTYPE, f"{name} must be {dtype}, got {x.dtype}")
    if shape is not None and tuple(x.shape) != tuple(shape):
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE, f"{name} has shape {tuple(x.shape)}, expected {tuple(shape)}")


def host_workspace_bytes(B: int, T: int, H: int, d: int, dtype: torch.dtype,
                         has_segment: bool = False) -> int:
    return int(capi.lib().rhz_gdr_host_workspace_bytes(B, T, H, d, _DTYPES[dtype],
                                                         1 if has_segment else 0))


def gdr_scan_chunked_host(q, k, v, alpha, beta, chunk=64, segment=None, state_init=None,
                          with_state=True, out=None, state_out=None, workspace=None,
                          device=None):
    """gated_delta_scan_chunked on HOST tensors [B, T, H, d] (pinned for the
    copies to overlap): the library copies slabs in, scans them on `device`
    and copies the outputs back, pipelined. Returns host (o, final|None)."""
    B, T = q.shape[0], q.shape[1]
    d, H = q.shape[-1], q.shape[-2]
    for name, x in (("q", q), ("k", k), ("v", v)):
        _need_host(x, name, q.dtype, (B, T, H, d))
    _need_host(alpha, "alpha", torch.float32, (B, T, H))
    _need_host(beta, "beta", torch.float32, (B, T, H))
    if segment is not None:
        _need_host(segment, "segment", torch.int64, (B, T))
    if state_init is not None:
        _need_host(state_init, "state_init", torch.float32, (B, H, d, d))
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    pin = q.is_pinned()
    o = out if out is not None else torch.empty(q.shape, dtype=q.dtype, pin_memory=pin)
    _need_host(o, "out", q.dtype, tuple(q.shape))
    fin = None
    if with_state:
        fin = state_out if state_out is not None else torch.empty((B, H, d, d), dtype=torch.float32,
                                                                  pin_memory=pin)
        _need_host(fin, "state_out", torch.float32, (B, H, d, d))
    nbytes = host_workspace_bytes(B, T, H, d, q.dtype, segment is not None)
    ws = workspace if workspace is not None else torch.empty(nbytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        capi.call("rhz_gdr_scan_chunked_host", _p(o), _p(fin), _p(q), _p(k), _p(v), _p(alpha),
                  _p(beta), _p(segment), _p(state_init), chunk, B, T, H, d, _dt(q), _p(ws),
                  ws.numel() * ws.element_size(), _stream(dev))
    return o, fin


def gdr_varlen_fwd(q, k, v, alpha, beta, cu_seqlens, state_pool=None, slot_idx=None,
                   zero_init=False, write_state=True, out=None, workspace=None):
    """Continuous-batching prefill over a packed stream q/k/v [tokens, H, d]:
    sequence i = rows [cu_seqlens[i], cu_seqlens[i+1]) resumes from
    state_pool[slot_idx[i]] (zeros if zero_init) and writes its final state
    back (if write_state). Returns o [tokens, H, d]."""
    tokens = q.shape[0]
    H, d = _qkv(q, k, v, alpha, beta, (tokens,))
    _need(cu_seqlens, "cu_seqlens", torch.int32)
    n_seq = cu_seqlens.numel() - 1
    flags = (capi.RHZ_FLAG_ZERO_INIT if zero_init else 0) | (0 if write_state else capi.RHZ_FLAG_NO_STATE_WRITE)
    num_slots = 0 if state_pool is None else _pool(state_pool, "state_pool", H, d)
    if slot_idx is not None:
        _need(slot_idx, "slot_idx", torch.int32, (n_seq,))
    if out is not None:
        _need(out, "out", q.dtype, tuple(q.shape))
    o = torch.empty_like(q) if out is None else out
    ws, nbytes = None, 0
    need = varlen_workspace_bytes(n_seq, H, d, q.dtype)
    if need > 0 or workspace is not None:
        ws, nbytes = _workspace(workspace, need, q.device)
    capi.call("rhz_gdr_varlen_fwd", _p(o), _p(state_pool), _p(slot_idx), _p(cu_seqlens), _p(q),
              _p(k), _p(v), _p(alpha), _p(beta), n_seq, tokens, num_slots, H, d, _dt(q), flags,
              _p(ws), nbytes, _stream(q.device))
    return o


def gdr_scan_chunked_bwd(q, k, v, alpha, beta, d_o, segment=None, d_state_final=None,
                         workspace=None):
    """Backward of gdr_scan_chunked / gdr_sequential on [B, T, H, d] (resets
    at t = 0 and at segment changes): returns (dq, dk, dv, dalpha, dbeta) for
    the upstream gradients d_o [B, T, H, d] and d_state_final [B, H, d, d]."""
    B, T = q.shape[0], q.shape[1]
    H, d = _qkv(q, k, v, alpha, beta, (B, T))
    _need(d_o, "d_o", q.dtype, tuple(q.shape))
    if segment is not None:
        _need(segment, "segment", torch.int64, (B, T))
    if d_state_final is not None:
        _need(d_state_final, "d_state_final", torch.float32, (B, H, d, d))
    ws, nbytes = _workspace(workspace, int(capi.lib().rhz_gdr_bwd_workspace_bytes(B, T, H, d)),
                            q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
    dalpha, dbeta = torch.empty_like(alpha), torch.empty_like(beta)
    capi.call("rhz_gdr_scan_chunked_bwd", _p(dq), _p(dk), _p(dv), _p(dalpha), _p(dbeta), _p(q),
              _p(k), _p(v), _p(alpha), _p(beta), _p(segment), _p(d_o), _p(d_state_final), B, T,
              H, d, _dt(q), _p(ws), nbytes, _stream(q.device))
    return dq, dk, dv, dalpha, dbeta


def gdr_varlen_fwd_norm(q, k, v, alpha, beta, cu_seqlens, norm_scale, norm_eps=1e-6,
                        state_pool=None, slot_idx=None, zero_init=False, write_state=True,
                        workspace=None):
    """gdr_varlen_fwd followed by the per-head output norm groupnorm_heads
    (norm.rs:48-60): each output row o[t, h] becomes
    o / sqrt(mean(o^2) + norm_eps) * norm_scale[:d]. Fused into the
    tensor-core kernel's epilogue on the bf16 d = 128 path."""
    tokens = q.shape[0]
    H, d = _qkv(q, k, v, alpha, beta, (tokens,))
    _need(cu_seqlens, "cu_seqlens", torch.int32)
    _need(norm_scale, "norm_scale", torch.float32)
    if norm_scale.numel() < d:
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE, f"norm_scale has {norm_scale.numel()} entries, need at least d = {d}")
    n_seq = cu_seqlens.numel() - 1
    flags = (capi.RHZ_FLAG_ZERO_INIT if zero_init else 0) | (0 if write_state else capi.RHZ_FLAG_NO_STATE_WRITE)
    num_slots = 0 if state_pool is None else _pool(state_pool, "state_pool", H, d)
    if slot_idx is not None:
        _need(slot_idx, "slot_idx", torch.int32, (n_seq,))
    o = torch.empty_like(q)
    ws, nbytes = None, 0
    need = varlen_workspace_bytes(n_seq, H, d, q.dtype)
    if need > 0 or workspace is not None:
        ws, nbytes = _workspace(workspace, need, q.device)
    capi.call("rhz_gdr_varlen_fwd_norm", _p(o), _p(state_pool), _p(slot_idx), _p(cu_seqlens),
              _p(q), _p(k), _p(v), _p(alpha), _p(beta), _p(norm_scale), float(norm_eps), n_seq,
              tokens, num_slots, H, d, _dt(q), flags, _p(ws), nbytes, _stream(q.device))
    return o


def groupnorm_heads(x, scale, eps=1e-6, out=None):
    """groupnorm_heads (norm.rs:48-60) on x [..., H, d]: each head's d values
    RMS-normalised with scale[:d]; out may be x (in place)."""
    _need(x, "x")
    _need(scale, "scale", torch.float32)
    H, d = x.shape[-2], x.shape[-1]
    if scale.numel() < d:
        raise capi.ShapeError(capi.RHZ_ERR_SHAPE, f"scale has {scale.numel()} entries, need at least d = {d}")
    rows = x.numel() // (H * d) if x.numel() else 0
    if out is not None:
        _need(out, "out", x.dtype, tuple(x.shape))
    o = torch.empty_like(x) if out is None else out
    capi.call("rhz_groupnorm_heads", _p(o), _p(x), _p(scale), rows, H, d, float(eps), _dt(x),
              _stream(x.device))
    return o


# ---------------------------------------------------------------- varlen helpers

def prefix_sum(lengths: torch.Tensor) -> torch.Tensor:
    _need(lengths, "lengths", torch.int32)
    cu = torch.empty(lengths.numel() + 1, device=lengths.device, dtype=torch.int32)
    capi.call("rhz_varlen_prefix_sum", _p(cu), _p(lengths), lengths.numel(), _stream(lengths.device))
    return cu


def segments_to_cu_seqlens(segment: torch.Tensor):
    """[B, T] int64 segment ids -> (cu_seqlens [B*T+1] int32 (first n_seg+1
    valid), n_seg int32[1]) on the device."""
    _need(segment, "segment", torch.int64)
    B, T = segment.shape
    cu = torch.zeros(B * T + 1, device=segment.device, dtype=torch.int32)
    n = torch.zeros(1, device=segment.device, dtype=torch.int32)
    nbytes = int(capi.lib().rhz_varlen_workspace_bytes(B * T))
    ws = torch.empty(nbytes, device=segment.device, dtype=torch.uint8)
    capi.call("rhz_varlen_segments_to_cu_seqlens", _p(cu), _p(n), _p(segment), B, T, _p(ws),
              nbytes, _stream(segment.device))
    return cu, n


def chunk_map(cu_seqlens: torch.Tensor, chunk: int = 64, max_chunks: int | None = None):
    _need(cu_seqlens, "cu_seqlens", torch.int32)
    n_seq = cu_seqlens.numel() - 1
    if max_chunks is None:
        total = int(cu_seqlens[-1].item()) if n_seq > 0 else 0
        max_chunks = total // chunk + n_seq + 1
    dev = cu_seqlens.device
    cs = torch.full((max_chunks,), -1, device=dev, dtype=torch.int32)
    st = torch.full((max_chunks,), -1, device=dev, dtype=torch.int32)
    n = torch.zeros(1, device=dev, dtype=torch.int32)
    nbytes = int(capi.lib().rhz_varlen_workspace_bytes(max(n_seq, 1)))
    ws = torch.empty(nbytes, device=dev, dtype=torch.uint8)
    capi.call("rhz_varlen_chunk_map", _p(cs), _p(st), _p(n), _p(cu_seqlens), n_seq, chunk,
              max_chunks, _p(ws), nbytes, _stream(dev))
    return cs, st, n


def gather_states(pool: torch.Tensor, slot_idx: torch.Tensor | None, n: int | None = None):
    _need(pool, "pool", torch.float32)
    S, H, d, _ = pool.shape
    n = slot_idx.numel() if slot_idx is not None else (n if n is not None else S)
    dense = torch.empty((n, H, d, d), device=pool.device, dtype=torch.float32)
    capi.call("rhz_varlen_gather_states", _p(dense), _p(pool), _p(slot_idx), n, S, H, d,
              _stream(pool.device))
    return dense


def scatter_states(pool: torch.Tensor, dense: torch.Tensor, slot_idx: torch.Tensor | None):
    _need(pool, "pool", torch.float32)
    _need(dense, "dense", torch.float32)
    S, H, d, _ = pool.shape
    n = dense.shape[0]
    capi.call("rhz_varlen_scatter_states", _p(pool), _p(dense), _p(slot_idx), n, S, H, d,
              _stream(pool.device))
    return pool


def pack_tokens(padded: torch.Tensor, cu_seqlens: torch.Tensor, total: int) -> torch.Tensor:
    """padded [n, max_len, ...] -> packed [total, ...] by cu_seqlens."""
    _need(padded, "padded")
    n, max_len = padded.shape[0], padded.shape[1]
    row_bytes = padded[0, 0].numel() * padded.element_size()
    packed = torch.zeros((total, *padded.shape[2:]), device=padded.device, dtype=padded.dtype)
    capi.call("rhz_varlen_pack_tokens", _p(packed), _p(padded), _p(cu_seqlens), n, max_len,
              row_bytes, _stream(padded.device))
    return packed


def unpack_tokens(packed: torch.Tensor, cu_seqlens: torch.Tensor, max_len: int) -> torch.Tensor:
    _need(packed, "packed")
    n = cu_seqlens.numel() - 1
    row_bytes = packed[0].numel() * packed.element_size() if packed.shape[0] else 4
    padded = torch.zeros((n, max_len, *packed.shape[1:]), device=packed.device, dtype=packed.dtype)
    capi.call("rhz_varlen_unpack_tokens", _p(padded), _p(packed), _p(cu_seqlens), n, max_len,
              row_bytes, _stream(packed.device))
    return padded


def device_status(clear: bool = False) -> bool:
    """True if a bounded device-side wait of a tensor-core kernel ran out on
    the current device since the last clear (that launch's outputs are
    undefined); ``clear`` resets the flag."""
    flag = ctypes.c_int32(0)
    capi.call("rhz_device_status", ctypes.byref(flag), 1 if clear else 0)
    return bool(flag.value)


def set_chunk_kernel(variant: str) -> str:
    """Pick the tensor-core chunked form process-wide: "auto" (the grid
    form), "grid" (chain CTAs fed by producer CTAs over every SM), "pair"
    (2-CTA cluster per item) or "solo" (one CTA per item). Returns the
    previous setting."""
    names = {"auto": capi.RHZ_CHUNK_AUTO, "pair": capi.RHZ_CHUNK_PAIR, "solo": capi.RHZ_CHUNK_SOLO,
             "grid": capi.RHZ_CHUNK_GRID}
    if variant not in names:
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"unknown chunk kernel {variant!r}")
    prev = ctypes.c_int32(0)
    capi.call("rhz_gdr_set_chunk_kernel", names[variant], ctypes.byref(prev))
    return {v: k for k, v in names.items()}[prev.value]


def set_bwd_kernel(variant: str) -> str:
    """Pick the backward's form process-wide: "auto" (the chunked
    tensor-core form for bf16, d = 128 without segments, the fp32 reverse
    scan otherwise) or "scan" (the fp32 reverse scan always). Returns the
    previous setting."""
    names = {"auto": capi.RHZ_BWD_AUTO, "scan": capi.RHZ_BWD_SCAN}
    if variant not in names:
        raise capi.InvalidArgument(capi.RHZ_ERR_INVALID, f"unknown backward kernel {variant!r}")
    prev = ctypes.c_int32(0)
    capi.call("rhz_gdr_set_bwd_kernel", names[variant], ctypes.byref(prev))
    return {v: k for k, v in names.items()}[prev.value]
