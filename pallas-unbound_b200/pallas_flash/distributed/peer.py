"""NVLink peer-memory exchange for the sequence-sharded decode.

Replaces the all-gather of the packed (m, l, o) partials
(`collectives.all_gather_partials`) with direct peer stores: every rank
allocates one exchange buffer (pu_peer_alloc), the IPC handles are shared
once over the process group, and each rank maps the others' buffers
(pu_peer_open).  A decode step is then one or two kernels per rank and no
collective: pu_decode_sharded (the split-KV pass stores each (b, h) record
into every rank's buffer as epoch-tagged words; a bounded wait for the G
records and the stable LogSumExp merge follow, inside the same kernel for
small B*H, else as a second kernel).  The merge the reference documents
for its sharded decode is a psum of LogSumExp terms (README.md:41-46).

All ranks must call `decode` the same number of times (the epoch counter
advances in lockstep); `close()` is collective.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional

import torch
import torch.distributed as dist

from .. import _lib

__all__ = ["PeerBuffers", "PeerExchange", "get_exchange", "get_cached", "close_all"]

IPC_HANDLE_BYTES = 64
DEFAULT_TIMEOUT_NS = 1_000_000_000  # 1 s


class PeerBuffers:
    """One zeroed, IPC-exportable device buffer per rank of `group`, mapped
    into every rank's address space (pu_peer_alloc / pu_peer_open).
    `ptrs[g]` is this process's pointer to rank g's buffer.  Collective."""

    def __init__(self, nbytes: int, group=None):
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if not 1 <= self.world <= 8:
            raise ValueError("peer buffers support 1..8 ranks")
        lib = _lib.lib()
        self.nbytes = int(nbytes)
        local = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _lib.check(lib.pu_peer_alloc(self.nbytes, ctypes.byref(local), handle), "pu_peer_alloc")
        self._local = local.value
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=self.group)
        ptrs = []
        self._opened = []
        try:
            for g, h in enumerate(handles):
                if g == self.rank:
                    ptrs.append(self._local)
                    continue
                p = ctypes.c_void_p()
                _lib.check(lib.pu_peer_open(ctypes.create_string_buffer(h, IPC_HANDLE_BYTES),
                                            ctypes.byref(p)), "pu_peer_open")
                ptrs.append(p.value)
                self._opened.append(p.value)
        except Exception:
            self._release()
            raise
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        self.epoch = 0
        # every rank has mapped every buffer before anyone stores into it
        dist.barrier(group=self.group)

    def next_epoch(self) -> int:
        self.epoch += 1
        if self.epoch >= 2 ** 31:
            raise RuntimeError("epoch counter exhausted; create new buffers")
        return self.epoch

    def _release(self):
        lib = _lib.lib()
        for p in self._opened:
            lib.pu_peer_close(p)
        self._opened = []
        if self._local:
            lib.pu_peer_free(self._local)
            self._local = None

    def close(self):
        """Collective: unmap and free once no rank can still store."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self._release()


class PeerExchange(PeerBuffers):
    """Exchange buffers of one process group for one (B, H, D) decode shape."""

    def __init__(self, B: int, H: int, D: int, group=None):
        g = group if group is not None else dist.group.WORLD
        self.B, self.H, self.D = B, H, D
        super().__init__(int(_lib.lib().pu_decode_exchange_bytes(B, H, D, dist.get_world_size(g))), g)

    def decode(self, q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor, *,
               kv_offset: int, kv_lens: Optional[torch.Tensor], sm_scale: float,
               workspace: torch.Tensor, timeout_ns: int = DEFAULT_TIMEOUT_NS):
        """One sharded decode step -> (o bf16 [B,H,1,D], lse fp32 [B,H]) on every rank."""
        from ..kernels.decoding import _DT
        B, H, D = self.B, self.H, self.D
        lib = _lib.lib()
        stream = torch.cuda.current_stream().cuda_stream
        self.next_epoch()
        n_local = k_shard.shape[2]
        o = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device=q.device)
        lse = torch.empty((B, H), dtype=torch.float32, device=q.device)
        _lib.check(lib.pu_decode_sharded(q.data_ptr(), _DT[q.dtype], k_shard.data_ptr(),
                                         v_shard.data_ptr(), _DT[k_shard.dtype],
                                         kv_lens.data_ptr() if kv_lens is not None else None,
                                         int(kv_offset), self._ptrs, self.world, self.rank,
                                         self.epoch, o.data_ptr(), lse.data_ptr(),
                                         workspace.data_ptr(), workspace.numel(), B, H, n_local, D,
                                         float(sm_scale), int(timeout_ns), stream),
                   "pu_decode_sharded")
        return o, lse



_cache: dict = {}
_cache_lock = threading.Lock()


def get_exchange(B: int, H: int, D: int, group=None) -> PeerExchange:
    """Cached PeerExchange per (group, device, B, H, D).  Collective on first use."""
    return get_cached(("decode", B, H, D), lambda: PeerExchange(B, H, D, group), group)


def get_cached(shape_key, make, group=None):
    """Cached peer buffers per (group, device, shape_key).  Collective on first use."""
    key = (id(group), torch.cuda.current_device()) + tuple(shape_key)
    with _cache_lock:
        ex = _cache.get(key)
    if ex is None:
        ex = make()
        with _cache_lock:
            _cache[key] = ex
    return ex


def close_all():
    """Collective: release every cached exchange (call before destroying the group)."""
    with _cache_lock:
        items = list(_cache.values())
        _cache.clear()
    for ex in items:
        ex.close()
