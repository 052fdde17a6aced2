"""Paged KV cache on the GPU (pu_decode_paged, pu_kv_append) against the
oracle's page gather and dense decode.

  * page_size 16 over the same cache length as the dense call: identical
    split plan, so the paged decode must equal pu_decode bit for bit
  * page sizes 32..256, D 64/128, fp16/bf16 mixes, ragged lengths (0, 1,
    page edges), pages in shuffled order: vs the oracle (o max-abs 2e-2 /
    rel 1e-2, LSE 1e-3)
  * append token by token into an empty cache: pools bit-exact with the
    appended values, lengths advanced on the device, then decode vs oracle
  * table entries outside the pool: reported through the device status word
    (detail 302 decode / 303 append), the rest of the batch still correct
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close_lse, assert_close_o
from oracle import attention as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods(built_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from pallas_flash import _lib
    from pallas_flash.kernels import decoding, paged
    _lib.device_status()  # clear any earlier status
    return _lib, decoding, paged


def _gen(shape, seed, dtype, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g) * scale).to(dtype)


def _f(t):
    return t.detach().float().cpu().numpy()


def test_paged_equals_dense_bitwise(mods):
    _lib, dec, paged = mods
    B, H, N, D, ps = 4, 8, 4096, 128, 16
    q = _gen((B, H, 1, D), 1, torch.float16)
    k = _gen((B, H, N, D), 2, torch.float16)
    v = _gen((B, H, N, D), 3, torch.float16)
    lens = torch.tensor([4096, 1, 2049, 0], dtype=torch.int32, device="cuda")
    o_d, l_d = dec.pallas_flash_decoding(q, k, v, kv_lens=lens, return_lse=True)
    cache = paged.PagedKVCache.from_dense(k, v, lens.cpu(), page_size=ps, shuffle_seed=5)
    assert cache.page_table.shape[1] * ps == N
    o_p, l_p = cache.decode(q, return_lse=True)
    torch.cuda.synchronize()
    assert _lib.device_status()[0] == 0
    assert torch.equal(o_p, o_d)
    assert torch.equal(l_p, l_d)


@pytest.mark.parametrize("ps,D,qdt,kvdt", [
    (32, 128, torch.float16, torch.float16),
    (64, 64, torch.bfloat16, torch.bfloat16),
    (128, 128, torch.bfloat16, torch.float16),
    (256, 128, torch.float16, torch.bfloat16),
])
def test_paged_decode_vs_oracle(mods, ps, D, qdt, kvdt):
    _lib, dec, paged = mods
    B, H, N = 5, 4, 3000
    q = _gen((B, H, 1, D), 10 + ps, qdt)
    k = _gen((B, H, N, D), 20 + ps, kvdt)
    v = _gen((B, H, N, D), 30 + ps, kvdt)
    lens = np.array([3000, ps, ps + 1, 1, 0], dtype=np.int32)
    cache = paged.PagedKVCache.from_dense(k, v, lens, page_size=ps, shuffle_seed=ps)
    o, lse = dec.pallas_flash_decoding(q, cache.k_pool, cache.v_pool, kv_lens=cache.kv_lens,
                                       page_table=cache.page_table, return_lse=True)
    torch.cuda.synchronize()
    assert _lib.device_status()[0] == 0
    kd = orc.paged_to_dense(_f(cache.k_pool), cache.alloc.table, lens, ps, n=N)
    vd = orc.paged_to_dense(_f(cache.v_pool), cache.alloc.table, lens, ps, n=N)
    np.testing.assert_array_equal(kd[0], _f(k[0]))
    ro, rl = orc.decode_forward(_f(q), kd, vd, kv_lens=lens)
    assert_close_o(_f(o), ro, what=f"paged decode ps={ps}")
    live = lens > 0
    assert_close_lse(_f(lse)[live], rl[live])
    assert (_f(o)[~live] == 0).all() and np.isneginf(_f(lse)[~live]).all()


def test_append_then_decode(mods):
    _lib, dec, paged = mods
    B, H, D, ps, T = 3, 8, 128, 32, 200
    cache = paged.PagedKVCache(B, H, D, num_pages=3 * 7 + 2, page_size=ps, max_seq_len=224,
                               dtype=torch.bfloat16)
    cache.alloc.shuffle(3)
    ks = _gen((T, B, H, 1, D), 40, torch.bfloat16)
    vs = _gen((T, B, H, 1, D), 41, torch.bfloat16)
    for t in range(T):
        cache.append(ks[t], vs[t])
    q = _gen((B, H, 1, D), 42, torch.bfloat16)
    o, lse = cache.decode(q, return_lse=True)
    torch.cuda.synchronize()
    assert _lib.device_status()[0] == 0
    assert cache.kv_lens.tolist() == [T] * B
    lens = np.full(B, T)
    kd = orc.paged_to_dense(_f(cache.k_pool), cache.alloc.table, lens, ps, n=T)
    vd = orc.paged_to_dense(_f(cache.v_pool), cache.alloc.table, lens, ps, n=T)
    kref = _f(ks)[:, :, :, 0].transpose(1, 2, 0, 3)
    vref = _f(vs)[:, :, :, 0].transpose(1, 2, 0, 3)
    np.testing.assert_array_equal(kd, kref)
    np.testing.assert_array_equal(vd, vref)
    ro, rl = orc.decode_forward(_f(q), kref, vref)
    assert_close_o(_f(o), ro, what="append then decode")
    assert_close_lse(_f(lse), rl)
    # releasing a sequence returns its pages and empties it
    free = cache.alloc.free_pages
    cache.release(1)
    assert cache.alloc.free_pages == free + 7 and cache.kv_lens.tolist() == [T, 0, T]


def test_invalid_page_entries_are_reported(mods):
    _lib, dec, paged = mods
    B, H, N, D, ps = 3, 4, 512, 128, 64
    q = _gen((B, H, 1, D), 50, torch.float16)
    k = _gen((B, H, N, D), 51, torch.float16)
    v = _gen((B, H, N, D), 52, torch.float16)
    lens = np.array([512, 300, 200], dtype=np.int32)
    cache = paged.PagedKVCache.from_dense(k, v, lens, page_size=ps)
    P = cache.k_pool.shape[0]
    # sequence 1: one entry past the pool, one negative
    bad = cache.page_table.clone()
    bad[1, 2] = P + 7
    bad[1, 4] = -3
    o = paged.paged_decode(q, cache.k_pool, cache.v_pool, bad, cache.kv_lens)
    code, detail = _lib.device_status()
    assert (code, detail) == (_lib.PU_ERR_INVALID_ARGUMENT, 302)
    ro, _ = orc.decode_forward(_f(q), _f(k), _f(v), kv_lens=lens)
    for b in (0, 2):
        assert_close_o(_f(o[b]), ro[b], what=f"valid sequence {b}")
    assert torch.isfinite(o.float()).all()
    # append: sequence 2's next slot (200 -> page 3) points outside the pool
    bad = cache.page_table.clone()
    bad[2, 3] = P
    before = cache.k_pool.clone()
    paged.kv_append(q, q, cache.k_pool, cache.v_pool, bad, cache.kv_lens)
    code, detail = _lib.device_status()
    assert (code, detail) == (_lib.PU_ERR_INVALID_ARGUMENT, 303)
    assert cache.kv_lens.tolist() == [512, 301, 200]
    changed = (cache.k_pool != before).any(dim=(1, 2, 3)).nonzero().flatten().tolist()
    assert changed == [int(cache.alloc.table[1, 300 // ps])]
    # sequence 0 is full (512 = 8 pages of 64): a further append is refused too
    assert cache.page_table.shape[1] == 8
