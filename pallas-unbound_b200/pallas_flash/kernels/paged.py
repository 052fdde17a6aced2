"""Paged KV cache for the decode path.

The reference's decode reads a dense, padded [B,H,N,D] cache
(src/pallas_flash/kernels/decoding.py:86-103) and has no cache update.  Here
the cache can also live in fixed-size pages, so sequences grow token by
token without re-allocating or copying:

  k_pool, v_pool  [num_pages, H, page_size, D]  fp16/bf16
  page_table      int32 [B, max_pages_per_seq]  physical page of each
                  logical page of a sequence (-1 = unmapped)
  kv_lens         int32 [B]                     tokens held per sequence

`paged_decode` (pu_decode_paged) gives the same result as
`pallas_flash_decoding` on the dense cache the pages describe;
`kv_append` (pu_kv_append) writes one token per sequence and advances
kv_lens on the device.  `PageAllocator` keeps the host-side free list and
table; `PagedKVCache` ties the pieces together.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

from .. import _lib
from .decoding import _DT, DecodeWorkspace

__all__ = ["PageAllocator", "PagedKVCache", "paged_decode", "kv_append"]


def _check_pool(k_pool: torch.Tensor, v_pool: torch.Tensor, page_table: torch.Tensor,
                kv_lens: torch.Tensor):
    if k_pool.shape != v_pool.shape or k_pool.dim() != 4:
        raise ValueError("k_pool and v_pool must both be [num_pages, H, page_size, D]")
    if k_pool.dtype != v_pool.dtype or k_pool.dtype not in _DT:
        raise ValueError("pools must share one dtype, fp16 or bf16")
    if page_table.dtype != torch.int32 or page_table.dim() != 2:
        raise ValueError("page_table must be int32 [B, max_pages_per_seq]")
    if kv_lens.dtype != torch.int32 or kv_lens.numel() != page_table.shape[0]:
        raise ValueError("kv_lens must be int32 [B]")
    for t in (k_pool, v_pool, page_table, kv_lens):
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("pools, page table and lengths must be contiguous CUDA tensors")


def paged_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                 page_table: torch.Tensor, kv_lens: torch.Tensor, *,
                 sm_scale: Optional[float] = None, return_lse: bool = False):
    """One decode step over a paged cache -> o bf16 [B,H,1,D] (and lse fp32 [B,H])."""
    _check_pool(k_pool, v_pool, page_table, kv_lens)
    P, H, page_size, D = k_pool.shape
    B, max_pages = page_table.shape
    if q.shape != (B, H, 1, D) or q.dtype not in _DT or not q.is_cuda:
        raise ValueError(f"q must be fp16/bf16 CUDA [{B}, {H}, 1, {D}]")
    q = q.contiguous()
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    lib = _lib.lib()
    o = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty((B, H), dtype=torch.float32, device=q.device)
    need = int(lib.pu_decode_paged_workspace_size(B, H, max_pages, page_size, D))
    ws = DecodeWorkspace.get(q.device, need)
    _lib.check(lib.pu_decode_paged(q.data_ptr(), _DT[q.dtype], k_pool.data_ptr(),
                                   v_pool.data_ptr(), _DT[k_pool.dtype], page_table.data_ptr(),
                                   max_pages, P, page_size, kv_lens.data_ptr(), o.data_ptr(),
                                   lse.data_ptr(), ws.data_ptr(), ws.numel(), B, H, D,
                                   float(sm_scale), torch.cuda.current_stream().cuda_stream),
               "pu_decode_paged")
    return (o, lse) if return_lse else o


def kv_append(k_new: torch.Tensor, v_new: torch.Tensor, k_pool: torch.Tensor,
              v_pool: torch.Tensor, page_table: torch.Tensor, kv_lens: torch.Tensor) -> None:
    """Write k_new/v_new [B,H,1,D] at position kv_lens[b] and advance kv_lens (on the device)."""
    _check_pool(k_pool, v_pool, page_table, kv_lens)
    P, H, page_size, D = k_pool.shape
    B, max_pages = page_table.shape
    for t in (k_new, v_new):
        if t.shape != (B, H, 1, D) or t.dtype != k_pool.dtype or not t.is_cuda:
            raise ValueError(f"new k/v must be CUDA {k_pool.dtype} [{B}, {H}, 1, {D}]")
    k_new, v_new = k_new.contiguous(), v_new.contiguous()
    _lib.check(_lib.lib().pu_kv_append(k_new.data_ptr(), v_new.data_ptr(), _DT[k_pool.dtype],
                                       k_pool.data_ptr(), v_pool.data_ptr(),
                                       page_table.data_ptr(), max_pages, P, page_size,
                                       kv_lens.data_ptr(), B, H, D,
                                       torch.cuda.current_stream().cuda_stream),
               "pu_kv_append")


class PageAllocator:
    """Host-side page bookkeeping: a free list over `num_pages` physical pages
    and the [batch, max_pages_per_seq] table (-1 where unmapped).

    `reserve(b, n)` maps pages so that sequence b can hold n tokens;
    `release(b)` returns its pages.  Pure host logic (no device calls)."""

    def __init__(self, num_pages: int, page_size: int, batch: int, max_pages_per_seq: int):
        if page_size < 16 or page_size & (page_size - 1):
            raise ValueError("page_size must be a power of two >= 16")
        self.num_pages = int(num_pages)
        self.page_size = int(page_size)
        self.table = np.full((batch, max_pages_per_seq), -1, dtype=np.int32)
        self.mapped = np.zeros(batch, dtype=np.int64)   # table entries in use per sequence
        self._free = list(range(self.num_pages - 1, -1, -1))

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def reserve(self, b: int, n_tokens: int) -> bool:
        """Map pages for tokens [0, n_tokens) of sequence b; True if the table changed."""
        need = -(-int(n_tokens) // self.page_size)
        if need > self.table.shape[1]:
            raise ValueError(f"sequence {b}: {n_tokens} tokens exceed "
                             f"{self.table.shape[1]} pages of {self.page_size}")
        have = int(self.mapped[b])
        if need <= have:
            return False
        if need - have > len(self._free):
            raise MemoryError(f"page pool exhausted ({self.num_pages} pages)")
        for i in range(have, need):
            self.table[b, i] = self._free.pop()
        self.mapped[b] = need
        return True

    def release(self, b: int) -> None:
        for i in range(int(self.mapped[b]) - 1, -1, -1):
            self._free.append(int(self.table[b, i]))
            self.table[b, i] = -1
        self.mapped[b] = 0

    def shuffle(self, seed: int) -> None:
        """Randomise the order in which free pages are handed out."""
        np.random.Generator(np.random.PCG64(seed)).shuffle(self._free)


class PagedKVCache:
    """A paged KV cache on one GPU: pools, device page table and lengths.

    cache = PagedKVCache(B, H, D, num_pages=..., page_size=64, max_seq_len=...)
    cache.append(k_new, v_new)       # one token per sequence
    o = cache.decode(q)              # attention of q over every held token
    """

    def __init__(self, batch: int, heads: int, head_dim: int, *, num_pages: int,
                 page_size: int = 64, max_seq_len: int, dtype=torch.bfloat16, device=None):
        if dtype not in _DT:
            raise ValueError("cache dtype must be fp16 or bf16")
        device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        max_pages = -(-int(max_seq_len) // page_size)
        self.alloc = PageAllocator(num_pages, page_size, batch, max_pages)
        self.k_pool = torch.zeros((num_pages, heads, page_size, head_dim), dtype=dtype, device=device)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.page_table = torch.from_numpy(self.alloc.table.copy()).to(device)
        self.kv_lens = torch.zeros(batch, dtype=torch.int32, device=device)
        self.host_lens = np.zeros(batch, dtype=np.int64)

    @property
    def page_size(self) -> int:
        return self.alloc.page_size

    def _push_table(self) -> None:
        self.page_table.copy_(torch.from_numpy(self.alloc.table))

    @classmethod
    def from_dense(cls, k: torch.Tensor, v: torch.Tensor, kv_lens, *, page_size: int = 64,
                   num_pages: Optional[int] = None, shuffle_seed: Optional[int] = None):
        """Pack dense caches [B,H,N,D] (first kv_lens[b] tokens of each sequence)."""
        B, H, N, D = k.shape
        lens = np.asarray(torch.as_tensor(kv_lens).cpu(), dtype=np.int64)
        pages_needed = int(sum(-(-int(n) // page_size) for n in lens))
        cache = cls(B, H, D, num_pages=num_pages or max(1, pages_needed), page_size=page_size,
                    max_seq_len=N, dtype=k.dtype, device=k.device)
        if shuffle_seed is not None:
            cache.alloc.shuffle(shuffle_seed)
        for b in range(B):
            n = int(lens[b])
            cache.alloc.reserve(b, n)
            for i in range(-(-n // page_size)):
                t0, t1 = i * page_size, min(n, (i + 1) * page_size)
                pg = int(cache.alloc.table[b, i])
                cache.k_pool[pg, :, :t1 - t0] = k[b, :, t0:t1]
                cache.v_pool[pg, :, :t1 - t0] = v[b, :, t0:t1]
        cache.host_lens[:] = lens
        cache.kv_lens.copy_(torch.from_numpy(lens.astype(np.int32)))
        cache._push_table()
        return cache

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Append one token [B,H,1,D] to every sequence, mapping pages as needed."""
        changed = False
        for b in range(self.host_lens.shape[0]):
            changed |= self.alloc.reserve(b, int(self.host_lens[b]) + 1)
        if changed:
            self._push_table()
        kv_append(k_new, v_new, self.k_pool, self.v_pool, self.page_table, self.kv_lens)
        self.host_lens += 1

    def release(self, b: int) -> None:
        """Drop sequence b and return its pages to the pool."""
        self.alloc.release(b)
        self.host_lens[b] = 0
        self.kv_lens[b] = 0
        self._push_table()

    def decode(self, q: torch.Tensor, *, sm_scale: Optional[float] = None,
               return_lse: bool = False):
        return paged_decode(q, self.k_pool, self.v_pool, self.page_table, self.kv_lens,
                            sm_scale=sm_scale, return_lse=return_lse)
