"""Decode entry point — drop-in for the reference's
`pallas_flash.kernels.decoding.pallas_flash_decoding`
(src/pallas_flash/kernels/decoding.py:105-145).

`pallas_flash_decoding(q, k_cache, v_cache)`: q [B,H,1,D], caches
[B,H,N,D]; returns bf16 [B,H,1,D] (the reference's output dtype).  The
reference casts every input to bf16 first (decoding.py:107-109); here fp16
and bf16 caches are read as they are (same bytes, no cast pass), other
dtypes are cast to bf16.

Keyword-only additions:
  kv_lens     int32 [B] per-sequence lengths (positions >= length masked,
              the reference's padding mask decoding.py:42-44 made ragged)
  sm_scale    default 1/sqrt(D)
  return_lse  also return fp32 LSE [B,H]
  group       a torch.distributed process group over which the cache is
              sharded by SEQUENCE: rank r holds tokens
              [r*N_local, (r+1)*N_local) of every sequence.  Each rank runs
              the split-KV kernel on its shard, the packed (m, l, o)
              partials are all-gathered over NCCL, and a fused stable-LSE
              kernel merges them (the split-KV scheme the reference documents,
              README.md:41-46, but never implements).
  sharding    for a sharded cache: "contiguous" (rank r holds positions
              [r*N_local, (r+1)*N_local) of every sequence; kv_lens are the
              global lengths) or "by_length" (rank r holds its slice of every
              sequence's held tokens from row 0 of its local cache, as
              distributed.collectives.length_balanced_split assigns them;
              kv_lens are this rank's local lengths), so a ragged batch keeps
              every rank equally busy
  transport   for a sharded cache: "nccl" (all-gather of the partials
              through torch.distributed), "lib" (the same all-gather through
              the library's own NCCL communicator, pu_allgather_partials) or
              "peer" (partials stored straight into every rank's exchange
              buffer over NVLink, flags instead of a collective; see
              distributed/peer.py)
  k_scale, v_scale  per-tensor scales of an fp8 (torch.float8_e4m3fn) cache:
              keys / values are the stored values times the scale
  page_table  int32 [B, max_pages_per_seq]: the caches are then page pools
              [num_pages, H, page_size, D] (see kernels/paged.py) and
              kv_lens is required; single GPU only.
"""
from __future__ import annotations

import math
import threading
from typing import Optional

import torch

from .. import _lib

__all__ = ["pallas_flash_decoding", "decode_partial", "decode_combine", "DecodeWorkspace"]

_DT = {torch.float16: _lib.PU_DTYPE_F16, torch.bfloat16: _lib.PU_DTYPE_BF16}
_FP8 = getattr(torch, "float8_e4m3fn", None)
_DT_KV = {**_DT, **({_FP8: _lib.PU_DTYPE_FP8_E4M3} if _FP8 is not None else {})}


class DecodeWorkspace:
    """Zero-initialised device scratch for the split-KV kernels, cached per
    (device, stream).  The kernels leave it zeroed after each call, so one
    workspace must not be shared by decode calls that overlap on the GPU."""

    _cache: dict = {}
    _lock = threading.Lock()

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        stream = torch.cuda.current_stream(device).cuda_stream
        key = (device.index, stream)
        with cls._lock:
            buf = cls._cache.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
                cls._cache[key] = buf
            return buf


def _prep(t: torch.Tensor, dev: torch.device, kinds=_DT) -> torch.Tensor:
    t = t.to(dev, non_blocking=True)
    if t.dtype not in kinds:
        t = t.to(torch.bfloat16)
    return t.contiguous()


def decode_partial(q, k_cache, v_cache, *, kv_offset: int = 0, kv_lens=None,
                   sm_scale: Optional[float] = None, out: Optional[torch.Tensor] = None):
    """Packed shard partial fp32 [B*H, D+2] = {m, l, o[D]} (pu_decode_partial)."""
    B, H, _, D = q.shape
    n_local = k_cache.shape[2]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B * H, D + 2), dtype=torch.float32, device=q.device)
    lib = _lib.lib()
    need = int(lib.pu_decode_workspace_size(B, H, n_local, D))
    ws = DecodeWorkspace.get(q.device, need)
    lens_ptr = kv_lens.data_ptr() if kv_lens is not None else None
    _lib.check(lib.pu_decode_partial(q.data_ptr(), _DT[q.dtype], k_cache.data_ptr(),
                                     v_cache.data_ptr(), _DT[k_cache.dtype], lens_ptr,
                                     int(kv_offset), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                     B, H, n_local, D, float(sm_scale),
                                     torch.cuda.current_stream().cuda_stream),
               "pu_decode_partial")
    return out


def decode_combine(parts: torch.Tensor, B: int, H: int, D: int, *, out=None, lse=None):
    """Merge gathered partials fp32 [G, B*H, D+2] -> (o bf16 [B,H,1,D], lse fp32 [B,H])."""
    G = parts.shape[0]
    if out is None:
        out = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device=parts.device)
    if lse is None:
        lse = torch.empty((B, H), dtype=torch.float32, device=parts.device)
    _lib.check(_lib.lib().pu_decode_combine(parts.data_ptr(), G, out.data_ptr(), lse.data_ptr(),
                                            B, H, D, torch.cuda.current_stream().cuda_stream),
               "pu_decode_combine")
    return out, lse


def pallas_flash_decoding(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                          kv_lens: Optional[torch.Tensor] = None,
                          sm_scale: Optional[float] = None, return_lse: bool = False,
                          group=None, transport: str = "nccl", sharding: str = "contiguous",
                          page_table: Optional[torch.Tensor] = None,
                          k_scale: float = 1.0, v_scale: float = 1.0):
    """One decode step of attention for a query token per (b, h)."""
    if page_table is not None:
        from .paged import paged_decode
        if group is not None or kv_lens is None:
            raise ValueError("a paged cache needs kv_lens and runs on one GPU (group=None)")
        return paged_decode(q, k_cache, v_cache, page_table, kv_lens, sm_scale=sm_scale,
                            return_lse=return_lse)
    if q.dim() != 4 or q.shape[2] != 1:
        raise ValueError("q must be [B, H, 1, D]")
    if k_cache.shape != v_cache.shape or k_cache.shape[0] != q.shape[0] \
            or k_cache.shape[3] != q.shape[3] or q.shape[1] % k_cache.shape[1] != 0:
        raise ValueError(f"cache shape {tuple(k_cache.shape)} does not match q {tuple(q.shape)}")
    H_kv = k_cache.shape[1]
    grouped = H_kv != q.shape[1] or k_cache.dtype == _FP8 or k_scale != 1.0 or v_scale != 1.0
    if grouped and (group is not None or page_table is not None):
        raise ValueError("grouped K/V heads and fp8 caches: single-GPU dense caches only")
    host = not q.is_cuda
    dev = torch.device("cuda", torch.cuda.current_device()) if host else q.device
    kinds = _DT_KV if grouped else _DT
    q_, k_, v_ = _prep(q, dev), _prep(k_cache, dev, kinds), _prep(v_cache, dev, kinds)
    B, H, _, D = q_.shape
    if D not in (64, 128):
        raise ValueError(f"decode head size {D} (supported: 64, 128)")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    lens = None
    if kv_lens is not None:
        lens = torch.as_tensor(kv_lens, dtype=torch.int32).to(dev, non_blocking=True).contiguous()
        if lens.numel() != B:
            raise ValueError("kv_lens must have B entries")
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    n_local = k_.shape[2]
    if grouped:
        o = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device=dev)
        lse = torch.empty((B, H), dtype=torch.float32, device=dev)
        ws = DecodeWorkspace.get(dev, int(lib.pu_decode_gqa_workspace_size(B, H, H_kv, n_local, D)))
        _lib.check(lib.pu_decode_gqa(q_.data_ptr(), _DT[q_.dtype], k_.data_ptr(), v_.data_ptr(),
                                     _DT_KV[k_.dtype],
                                     lens.data_ptr() if lens is not None else None,
                                     o.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), B, H,
                                     H_kv, n_local, D, float(sm_scale), float(k_scale),
                                     float(v_scale), stream), "pu_decode_gqa")
    elif group is None:
        o = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device=dev)
        lse = torch.empty((B, H), dtype=torch.float32, device=dev)
        need = int(lib.pu_decode_workspace_size(B, H, n_local, D))
        ws = DecodeWorkspace.get(dev, need)
        _lib.check(lib.pu_decode(q_.data_ptr(), _DT[q_.dtype], k_.data_ptr(), v_.data_ptr(),
                                 _DT[k_.dtype], lens.data_ptr() if lens is not None else None,
                                 o.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), B, H,
                                 n_local, D, float(sm_scale), stream), "pu_decode")
    else:
        import torch.distributed as dist
        rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        if sharding == "contiguous":
            kv_offset = rank * n_local
        elif sharding == "by_length":
            if lens is None:
                raise ValueError('sharding="by_length" needs this rank\'s kv_lens')
            kv_offset = 0
        else:
            raise ValueError(f"unknown sharding {sharding!r} (contiguous or by_length)")
        if transport == "peer":
            from ..distributed.peer import get_exchange
            ex = get_exchange(B, H, D, group)
            ws = DecodeWorkspace.get(dev, int(lib.pu_decode_workspace_size(B, H, n_local, D)))
            o, lse = ex.decode(q_, k_, v_, kv_offset=kv_offset, kv_lens=lens,
                               sm_scale=sm_scale, workspace=ws)
        elif transport in ("nccl", "lib"):
            from ..distributed.collectives import all_gather_partials, get_lib_comm
            part = decode_partial(q_, k_, v_, kv_offset=kv_offset, kv_lens=lens,
                                  sm_scale=sm_scale)
            if transport == "nccl":
                gathered = all_gather_partials(part, world, group)
            else:
                gathered = get_lib_comm(group).all_gather(part, B, H, D)
            o, lse = decode_combine(gathered, B, H, D)
        else:
            raise ValueError(f"unknown transport {transport!r} (nccl, lib or peer)")
    if host:
        o, lse = o.cpu(), lse.cpu()
    return (o, lse) if return_lse else o
