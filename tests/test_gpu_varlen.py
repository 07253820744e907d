"""Bit-exact checks of the variable-length packing kernels (index and byte
work) against plain numpy on the same seeded inputs."""
import numpy as np
import pytest
import torch

from rhizome_b200 import ops
from tests.gpu_util import to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [0, 1, 5, 4095, 4096, 4097, 100_000])
def test_prefix_sum(n):
    rng = np.random.default_rng(n)
    lens = rng.integers(0, 9000, size=n).astype(np.int32)
    if n:
        lens[rng.integers(0, n, size=max(1, n // 10))] = 0
    cu = ops.prefix_sum(to_dev(lens, torch.int32))
    ref = np.concatenate([[0], np.cumsum(lens, dtype=np.int64)]).astype(np.int32)
    assert np.array_equal(cu.cpu().numpy(), ref)


def np_segments_to_cu(seg):
    B, T = seg.shape
    flat = seg.reshape(-1)
    flags = np.zeros(B * T, dtype=bool)
    flags[::T] = True
    flags[1:] |= flat[1:] != flat[:-1]
    starts = np.nonzero(flags)[0]
    return np.concatenate([starts, [B * T]]).astype(np.int32)


@pytest.mark.parametrize("B,T,p", [(1, 1, 0.0), (2, 10, 0.3), (4, 4096, 0.01), (3, 5000, 0.5),
                                   (1, 70_000, 0.001)])
def test_segments_to_cu_seqlens(B, T, p):
    rng = np.random.default_rng(B * T)
    seg = np.cumsum(rng.random((B, T)) < p, axis=1).astype(np.int64)
    seg[:, ::7] += 0  # ids are arbitrary int64; only changes matter
    if B > 1:
        seg[1] = seg[0]  # identical ids across rows still split at the row start
    cu, n = ops.segments_to_cu_seqlens(to_dev(seg, torch.int64))
    ref = np_segments_to_cu(seg)
    n = int(n.item())
    assert n == ref.size - 1
    assert np.array_equal(cu.cpu().numpy()[: n + 1], ref)


def test_segments_reference_fixture():
    """The segment pattern of delta.rs:305-317."""
    seg = np.array([[0, 0, 0, 1, 1, 2, 2, 2, 2, 3]], dtype=np.int64)
    cu, n = ops.segments_to_cu_seqlens(to_dev(seg, torch.int64))
    assert int(n.item()) == 4
    assert cu.cpu().numpy()[:5].tolist() == [0, 3, 5, 9, 10]


def np_chunk_map(cu, chunk):
    seqs, starts = [], []
    for i in range(cu.size - 1):
        for s in range(cu[i], cu[i + 1], chunk):
            seqs.append(i)
            starts.append(s)
    return np.array(seqs, np.int32), np.array(starts, np.int32)


@pytest.mark.parametrize("chunk", [1, 3, 64])
def test_chunk_map(chunk):
    rng = np.random.default_rng(chunk)
    lens = rng.integers(0, 300, size=700)
    lens[::5] = 0
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    cs, st, n = ops.chunk_map(to_dev(cu, torch.int32), chunk)
    rs, rst = np_chunk_map(cu, chunk)
    n = int(n.item())
    assert n == rs.size
    assert np.array_equal(cs.cpu().numpy()[:n], rs)
    assert np.array_equal(st.cpu().numpy()[:n], rst)


def test_chunk_map_truncates_but_reports_count():
    cu = np.array([0, 100, 250], dtype=np.int32)
    cs, st, n = ops.chunk_map(to_dev(cu, torch.int32), 64, max_chunks=3)
    assert int(n.item()) == 2 + 3
    assert cs.cpu().tolist() == [0, 0, 1] and st.cpu().tolist() == [0, 64, 100]


@pytest.mark.parametrize("d", [3, 32, 128])
def test_gather_scatter_states_bit_exact(d):
    S, H, n = 40, 3, 17
    g = torch.Generator(device="cuda").manual_seed(d)
    pool = torch.randn((S, H, d, d), device="cuda", generator=g)
    slots = torch.randperm(S, device="cuda", generator=g)[:n].to(torch.int32)
    dense = ops.gather_states(pool, slots)
    assert torch.equal(dense, pool[slots.long()])
    new = torch.randn_like(dense)
    before = pool.clone()
    ops.scatter_states(pool, new, slots)
    expect = before.clone()
    expect[slots.long()] = new
    assert torch.equal(pool, expect)


@pytest.mark.parametrize("row_elems,dtype", [(16 * 128, torch.bfloat16), (3, torch.float32),
                                             (16, torch.float32)])
def test_pack_unpack_tokens_bit_exact(row_elems, dtype):
    rng = np.random.default_rng(row_elems)
    n, max_len = 9, 50
    lens = rng.integers(0, max_len + 1, size=n)
    lens[0] = 0
    lens[1] = max_len
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    padded = torch.randn((n, max_len, row_elems), device="cuda").to(dtype)
    packed = ops.pack_tokens(padded, to_dev(cu, torch.int32), int(cu[-1]))
    ref = torch.cat([padded[i, : lens[i]] for i in range(n)])
    assert torch.equal(packed, ref)
    back = ops.unpack_tokens(packed, to_dev(cu, torch.int32), max_len)
    for i in range(n):
        assert torch.equal(back[i, : lens[i]], padded[i, : lens[i]])
        assert not back[i, lens[i]:].any()
