"""GPU parity of the split-KV decode kernels (pu_decode, pu_decode_partial,
pu_decode_combine) against the oracle's restatement of the reference's
decode (benchmarks/inference_decode.py:32-44, kernels/decoding.py:19-60)."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import assert_close_lse, assert_close_o, randn, to_np
from oracle import attention as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dec(built_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from pallas_flash.kernels import decoding
    return decoding


def _inputs(B, H, N, D, seed, dtype=torch.float16):
    q = randn((B, H, 1, D), seed, dtype=dtype)
    k = randn((B, H, N, D), seed + 1, dtype=dtype)
    v = randn((B, H, N, D), seed + 2, dtype=dtype)
    return q, k, v


@pytest.mark.parametrize("B,H,N,D,dtype", [(1, 4, 4096, 128, torch.float16),
                                           (2, 3, 1000, 128, torch.float16),
                                           (1, 2, 77, 128, torch.bfloat16),
                                           (2, 2, 5000, 64, torch.float16),
                                           (1, 1, 1, 128, torch.float16)])
def test_decode_single_gpu(dec, B, H, N, D, dtype):
    q, k, v = _inputs(B, H, N, D, 3, dtype)
    o, lse = dec.pallas_flash_decoding(q.cuda(), k.cuda(), v.cuda(), return_lse=True)
    torch.cuda.synchronize()
    assert o.shape == (B, H, 1, D) and o.dtype == torch.bfloat16
    ro, rl = orc.decode_forward(to_np(q), to_np(k), to_np(v))
    assert_close_o(to_np(o), ro)
    assert_close_lse(to_np(lse), rl)


def test_decode_ragged_lengths(dec):
    B, H, N, D = 4, 2, 3000, 128
    q, k, v = _inputs(B, H, N, D, 4)
    lens = torch.tensor([3000, 1, 128, 2177], dtype=torch.int32)
    o, lse = dec.pallas_flash_decoding(q.cuda(), k.cuda(), v.cuda(), kv_lens=lens.cuda(),
                                       return_lse=True)
    ro, rl = orc.decode_forward(to_np(q), to_np(k), to_np(v), kv_lens=lens.numpy())
    assert_close_o(to_np(o), ro)
    assert_close_lse(to_np(lse), rl)


@pytest.mark.parametrize("G", [2, 4, 8])
def test_decode_sharded_combine(dec, G):
    """Sequence shards -> per-shard partials -> stable LSE combine == whole cache."""
    B, H, N, D = 2, 4, 8192, 128
    q, k, v = _inputs(B, H, N, D, 5)
    lens = torch.tensor([8192, 3000], dtype=torch.int32)
    qc, kc, vc, lc = q.cuda(), k.cuda(), v.cuda(), lens.cuda()
    n_local = N // G
    parts = []
    for r in range(G):
        ks = kc[:, :, r * n_local:(r + 1) * n_local].contiguous()
        vs = vc[:, :, r * n_local:(r + 1) * n_local].contiguous()
        p = dec.decode_partial(qc, ks, vs, kv_offset=r * n_local, kv_lens=lc)
        ep = orc.decode_partial(to_np(q), to_np(k)[:, :, r * n_local:(r + 1) * n_local],
                                to_np(v)[:, :, r * n_local:(r + 1) * n_local],
                                kv_offset=r * n_local, kv_lens=lens.numpy())
        pn = to_np(p)
        # empty shards must report m = -inf, l = 0
        np.testing.assert_array_equal(np.isneginf(pn[:, 0]), np.isneginf(ep[:, 0]))
        parts.append(p)
    o, lse = dec.decode_combine(torch.stack(parts), B, H, D)
    ro, rl = orc.decode_forward(to_np(q), to_np(k), to_np(v), kv_lens=lens.numpy())
    assert_close_o(to_np(o), ro)
    assert_close_lse(to_np(lse), rl)


@pytest.mark.parametrize("G", [2, 4, 8])
def test_decode_length_balanced_shards(dec, G):
    """Length-balanced shards (every rank a slice of every sequence's held
    tokens, read with local lengths and no offset), one partial per shard,
    stable combine == the whole ragged cache."""
    from pallas_flash.distributed import collectives
    B, H, N, D = 4, 4, 6144, 128
    q, k, v = _inputs(B, H, N, D, 15)
    lens = np.array([6144, 4097, 128, 1])
    parts = []
    for r in range(G):
        kl, vl, ll = collectives.shard_by_length(k, v, lens, r, G, granule=128)
        parts.append(dec.decode_partial(q.cuda(), kl.cuda(), vl.cuda(), kv_offset=0, kv_lens=ll.cuda()))
    o, lse = dec.decode_combine(torch.stack(parts), B, H, D)
    ro, rl = orc.decode_forward(to_np(q), to_np(k), to_np(v), kv_lens=lens)
    assert_close_o(to_np(o), ro)
    assert_close_lse(to_np(lse), rl)


def test_decode_c4_full_size(dec):
    """B=1 H=32, 32768-token fp16 cache, D=128 (the split-KV decode benchmark shape)."""
    B, H, N, D = 1, 32, 32768, 128
    q, k, v = _inputs(B, H, N, D, 3)
    o, lse = dec.pallas_flash_decoding(q.cuda(), k.cuda(), v.cuda(), return_lse=True)
    ro, rl = orc.decode_forward(to_np(q), to_np(k), to_np(v), dtype=np.float64)
    assert_close_o(to_np(o), ro)
    assert_close_lse(to_np(lse), rl)


def test_decode_workspace_stays_zero(dec):
    """The kernel resets its arrival counters: repeated calls agree exactly."""
    q, k, v = _inputs(1, 8, 2048, 128, 6)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    a = dec.pallas_flash_decoding(qc, kc, vc)
    b = dec.pallas_flash_decoding(qc, kc, vc)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    from pallas_flash import _lib
    assert _lib.device_status()[0] == 0


def test_decode_emulates_reference_bf16_cast(dec):
    """Against the reference kernel's bf16 cast of fp16 inputs (decoding.py:107-109)."""
    q, k, v = _inputs(1, 4, 1024, 128, 8)
    o = dec.pallas_flash_decoding(q.cuda(), k.cuda(), v.cuda())
    qb, kb, vb = (orc.bf16_round(to_np(t)) for t in (q, k, v))
    ro, _ = orc.decode_forward(qb, kb, vb)
    assert_close_o(to_np(o), ro)
