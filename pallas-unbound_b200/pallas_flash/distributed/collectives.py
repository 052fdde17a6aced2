"""Cross-rank exchange of split-KV partials.

The reference's collectives (src/pallas_flash/distributed/collectives.py:27-117)
are XLA psum/all_gather wrappers that no kernel calls; its documented
split-KV merge is a psum of LogSumExp terms (README.md:41-46).  Here the one
real exchange step of the sequence-sharded decode is an NCCL all-gather of
the packed fp32 (m, l, o) records over NVLink, through torch.distributed
(backend "nccl" on GPUs, "gloo" in the CPU tests), or through the library's
own NCCL communicator (`LibComm`: pu_comm_* / pu_allgather_partials), the
route a caller without torch.distributed (a C or JAX FFI runtime) takes.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .. import _lib


def all_gather_partials(part: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """[BH, D+2] per rank -> [world, BH, D+2] on every rank (rank order)."""
    part = part.contiguous()
    out = torch.empty((world,) + tuple(part.shape), dtype=part.dtype, device=part.device)
    if dist.get_backend(group) == "gloo" or not hasattr(dist, "all_gather_into_tensor"):
        dist.all_gather(list(out.unbind(0)), part, group=group)
    else:
        dist.all_gather_into_tensor(out, part, group=group)
    return out


def sequence_shard(x: torch.Tensor, rank: int, world: int, axis: int = 2) -> torch.Tensor:
    """Contiguous sequence chunk `rank` of `world` (the cache sharding of the
    split-KV decode).  The sequence length must divide evenly."""
    n = x.shape[axis]
    if n % world:
        raise ValueError(f"sequence length {n} is not divisible by {world} shards")
    step = n // world
    return x.narrow(axis, rank * step, step)


def length_balanced_split(lens, world: int, granule: int = 128):
    """Sequence sharding by held tokens: rank r takes a contiguous slice of
    every sequence b, of about lens[b] / world tokens, so each rank reads the
    same number of K/V bytes however ragged the batch is (contiguous chunks of
    the padded capacity leave the high ranks idle past every sequence's end).

    Slices are whole `granule`-token blocks except the last block of a
    sequence; the blocks left over by the integer split go to the ranks
    (r - b) mod world < remainder, so the extra blocks rotate over ranks and
    no rank collects one from every sequence.

    Returns (starts, counts): int64 arrays [world, B]; rank r holds tokens
    [starts[r, b], starts[r, b] + counts[r, b]) of sequence b.
    """
    import numpy as np
    lens = np.asarray(lens, dtype=np.int64).reshape(-1)
    if world < 1 or granule < 1 or (lens < 0).any():
        raise ValueError("world and granule must be positive, lengths non-negative")
    B = lens.shape[0]
    blocks = (lens + granule - 1) // granule
    base, rem = blocks // world, blocks % world
    r = np.arange(world)[:, None]
    b = np.arange(B)[None, :]
    nblk = base[None, :] + (((r - b) % world) < rem[None, :]).astype(np.int64)
    first = np.concatenate([np.zeros((1, B), dtype=np.int64), np.cumsum(nblk, axis=0)[:-1]], axis=0)
    starts = np.minimum(first * granule, lens[None, :])
    ends = np.minimum((first + nblk) * granule, lens[None, :])
    return starts, ends - starts


def shard_by_length(k_cache: torch.Tensor, v_cache: torch.Tensor, lens, rank: int, world: int,
                    granule: int = 128, capacity: int | None = None):
    """This rank's length-balanced shard of full caches [B, H, N, D]: local
    caches [B, H, capacity, D] holding its slice of every sequence from row 0
    (rows past the slice are zero), and the local lengths int32 [B].
    `capacity` defaults to the longest local slice rounded up to `granule`."""
    starts, counts = length_balanced_split(lens, world, granule)
    st, ct = starts[rank], counts[rank]
    cap = capacity if capacity is not None else max(granule, int(-(-int(ct.max()) // granule) * granule))
    B, H, _, D = k_cache.shape
    kl = torch.zeros((B, H, cap, D), dtype=k_cache.dtype, device=k_cache.device)
    vl = torch.zeros_like(kl)
    for b in range(B):
        n = int(ct[b])
        if n:
            kl[b, :, :n] = k_cache[b, :, int(st[b]):int(st[b]) + n]
            vl[b, :, :n] = v_cache[b, :, int(st[b]):int(st[b]) + n]
    return kl, vl, torch.as_tensor(ct, dtype=torch.int32)


class LibComm:
    """The library's own NCCL communicator over the ranks of `group` (the
    group only carries the unique id from rank 0 to the others).  One per
    (group, device); `all_gather` runs pu_allgather_partials on the current
    stream."""

    def __init__(self, group=None):
        g = group if group is not None else dist.group.WORLD
        self.rank, self.world = dist.get_rank(g), dist.get_world_size(g)
        lib = _lib.lib()
        uid = (ctypes.c_uint8 * _lib.PU_COMM_ID_BYTES)()
        if self.rank == 0:
            _lib.check(lib.pu_comm_unique_id(uid), "pu_comm_unique_id")
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=dist.get_global_rank(g, 0), group=g)
        uid = (ctypes.c_uint8 * _lib.PU_COMM_ID_BYTES).from_buffer_copy(box[0])
        self._comm = ctypes.c_void_p()
        _lib.check(lib.pu_comm_init(uid, self.world, self.rank, ctypes.byref(self._comm)), "pu_comm_init")

    def all_gather(self, part: torch.Tensor, B: int, H: int, D: int) -> torch.Tensor:
        """fp32 [B*H, D+2] of this rank -> [world, B*H, D+2] on every rank."""
        if part.dtype != torch.float32 or tuple(part.shape) != (B * H, D + 2) or not part.is_cuda:
            raise TypeError(f"partial must be a CUDA fp32 [{B * H}, {D + 2}] tensor, got "
                            f"{part.dtype} {tuple(part.shape)} on {part.device}")
        part = part.contiguous()
        out = torch.empty((self.world,) + tuple(part.shape), dtype=torch.float32, device=part.device)
        _lib.check(_lib.lib().pu_allgather_partials(part.data_ptr(), out.data_ptr(), B, H, D, self._comm,
                                                    torch.cuda.current_stream().cuda_stream),
                   "pu_allgather_partials")
        return out

    def close(self):
        if self._comm:
            _lib.check(_lib.lib().pu_comm_destroy(self._comm), "pu_comm_destroy")
            self._comm = ctypes.c_void_p()


_COMMS: dict = {}


def get_lib_comm(group=None) -> LibComm:
    """The cached LibComm of (group, current device); built collectively on first use."""
    key = (id(group), torch.cuda.current_device())
    if key not in _COMMS:
        _COMMS[key] = LibComm(group)
    return _COMMS[key]


def close_lib_comms():
    for c in _COMMS.values():
        c.close()
    _COMMS.clear()
