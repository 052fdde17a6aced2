"""Cross-rank exchange of split-KV partials.

The reference's collectives (src/pallas_flash/distributed/collectives.py:27-117)
are XLA psum/all_gather wrappers that no kernel calls; its documented
split-KV merge is a psum of LogSumExp terms (README.md:41-46).  Here the one
real exchange step of the sequence-sharded decode is an NCCL all-gather of
the packed fp32 (m, l, o) records over NVLink, through torch.distributed
(backend "nccl" on GPUs, "gloo" in the CPU tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


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
