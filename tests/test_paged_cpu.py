"""Paged KV cache on the CPU: the oracle's page gather/append, the host page
allocator, and argument errors of the paged entry points (no GPU calls)."""
from __future__ import annotations

import numpy as np
import pytest

from helpers import randn as _randn
from oracle import attention as orc


def randn(shape, seed):
    return _randn(shape, seed).float().numpy()


def _pack(k, lens, page_size, rng):
    """Dense [B,H,N,D] -> (pool, table) with pages handed out in random order."""
    B, H, N, D = k.shape
    need = [-(-int(n) // page_size) for n in lens]
    P = sum(need) + 3
    order = rng.permutation(P)
    pool = np.zeros((P, H, page_size, D), dtype=k.dtype)
    table = np.full((B, -(-N // page_size)), -1, dtype=np.int32)
    nxt = 0
    for b in range(B):
        for i in range(need[b]):
            pg = int(order[nxt]); nxt += 1
            table[b, i] = pg
            t0, t1 = i * page_size, min(int(lens[b]), (i + 1) * page_size)
            pool[pg, :, :t1 - t0] = k[b, :, t0:t1]
    return pool, table


@pytest.mark.parametrize("page_size", [16, 64, 256])
def test_paged_round_trip(page_size):
    rng = np.random.Generator(np.random.PCG64(11))
    B, H, N, D = 3, 2, 700, 64
    k = randn((B, H, N, D), 1)
    lens = np.array([700, 1, 333])
    pool, table = _pack(k, lens, page_size, rng)
    dense = orc.paged_to_dense(pool, table, lens, page_size, n=N)
    for b in range(B):
        np.testing.assert_array_equal(dense[b, :, :lens[b]], k[b, :, :lens[b]])
        assert not dense[b, :, lens[b]:].any()


def test_paged_decode_matches_dense_oracle():
    rng = np.random.Generator(np.random.PCG64(12))
    B, H, N, D, ps = 2, 3, 300, 64, 32
    q, k, v = (randn(s, i) for i, s in enumerate([(B, H, 1, D), (B, H, N, D), (B, H, N, D)]))
    lens = np.array([300, 45])
    kp, table = _pack(k, lens, ps, rng)
    rng = np.random.Generator(np.random.PCG64(12))
    vp, table2 = _pack(v, lens, ps, rng)
    assert (table == table2).all()
    o1, l1 = orc.decode_forward(q, k, v, kv_lens=lens)
    o2, l2 = orc.decode_forward(q, orc.paged_to_dense(kp, table, lens, ps),
                                orc.paged_to_dense(vp, table, lens, ps), kv_lens=lens)
    np.testing.assert_array_equal(o1, o2)
    np.testing.assert_array_equal(l1, l2)


def test_paged_append_sequence():
    """Appending tokens one at a time reproduces the dense cache; sequences
    whose next slot has no valid page are left unchanged."""
    B, H, D, ps, T = 3, 2, 8, 16, 40
    P = 12
    kp = np.zeros((P, H, ps, D), np.float32)
    vp = np.zeros_like(kp)
    table = np.array([[5, 0, 7], [1, 2, 3], [4, 99, -1]], dtype=np.int32)  # seq 2: bad 2nd page
    lens = np.zeros(B, np.int64)
    ks = randn((T, B, H, 1, D), 3)
    vs = randn((T, B, H, 1, D), 4)
    for t in range(T):
        lens = orc.paged_append(kp, vp, table, lens, ks[t], vs[t], ps)
    assert list(lens) == [40, 40, 16]
    dk = orc.paged_to_dense(kp, table, lens, ps)
    dv = orc.paged_to_dense(vp, table, lens, ps)
    for b in range(B):
        n = int(lens[b])
        np.testing.assert_array_equal(dk[b, :, :n], ks[:n, b, :, 0].transpose(1, 0, 2))
        np.testing.assert_array_equal(dv[b, :, :n], vs[:n, b, :, 0].transpose(1, 0, 2))


def test_page_allocator():
    from pallas_flash.kernels.paged import PageAllocator
    a = PageAllocator(num_pages=6, page_size=16, batch=2, max_pages_per_seq=4)
    assert a.reserve(0, 1) and not a.reserve(0, 16) and a.reserve(0, 17)
    assert a.mapped.tolist() == [2, 0] and a.free_pages == 4
    assert a.reserve(1, 64) and a.free_pages == 0
    with pytest.raises(MemoryError):
        a.reserve(0, 33)
    with pytest.raises(ValueError):
        a.reserve(1, 65)
    used = set(a.table[0, :2]) | set(a.table[1])
    assert used == set(range(6))
    a.release(1)
    assert a.free_pages == 4 and (a.table[1] == -1).all()
    assert a.reserve(0, 64) and a.mapped[0] == 4
    with pytest.raises(ValueError):
        PageAllocator(4, 24, 1, 1)


def test_paged_argument_errors_without_gpu(built_lib):
    from pallas_flash import _lib
    lib = _lib.lib()
    dummy = 1 << 12  # never dereferenced: the host checks reject the call first
    # page size not a power of two
    rc = lib.pu_decode_paged(dummy, _lib.PU_DTYPE_BF16, dummy, dummy, _lib.PU_DTYPE_BF16, dummy,
                             4, 8, 24, dummy, dummy, None, dummy, 1 << 20, 1, 1, 128, 0.1, None)
    assert rc == _lib.PU_ERR_UNSUPPORTED and b"page size" in lib.pu_last_error()
    # null page table
    rc = lib.pu_kv_append(dummy, dummy, _lib.PU_DTYPE_F16, dummy, dummy, None, 4, 8, 16, dummy,
                          1, 1, 128, None)
    assert rc == _lib.PU_ERR_INVALID_ARGUMENT and b"page table" in lib.pu_last_error()
    # unsupported cache dtype
    rc = lib.pu_kv_append(dummy, dummy, _lib.PU_DTYPE_F32, dummy, dummy, dummy, 4, 8, 16, dummy,
                          1, 1, 128, None)
    assert rc == _lib.PU_ERR_UNSUPPORTED
    assert lib.pu_decode_paged_workspace_size(0, 1, 1, 16, 128) == 0
