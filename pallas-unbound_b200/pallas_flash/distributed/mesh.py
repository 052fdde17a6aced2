"""Head/batch partitioning of the training attention across GPUs.

Mirror of the reference's src/pallas_flash/distributed/mesh.py:31-92: a 2-D
('dp', 'tp') mesh where [B, H, N, D] tensors are partitioned as
P('dp', 'tp', None, None) — batch over dp, heads over tp (mesh.py:57-77).
On B200 each rank is one process owning one GPU; the partition is computed
per rank and the attention kernels run on the local slice with no
collective (heads and batch entries are independent).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Mesh:
    dp: int
    tp: int

    @property
    def size(self) -> int:
        return self.dp * self.tp

    def coords(self, rank: int) -> tuple[int, int]:
        """(dp_index, tp_index) of a rank (row-major, like the reference's reshape)."""
        if not 0 <= rank < self.size:
            raise ValueError(f"rank {rank} outside a {self.dp}x{self.tp} mesh")
        return rank // self.tp, rank % self.tp


def create_mesh(world_size: int, dp_size: int = 1, tp_size: int | None = None) -> Mesh:
    """Mesh over `world_size` ranks; falls back to 1 x world_size when the
    requested shape does not fit, as create_v5e_mesh does (mesh.py:44-50)."""
    if tp_size is None:
        tp_size = world_size // max(dp_size, 1)
    if dp_size * tp_size > world_size or dp_size * tp_size == 0:
        dp_size, tp_size = 1, world_size
    return Mesh(dp_size, tp_size)


def shard_bounds(n: int, parts: int, index: int) -> tuple[int, int]:
    if n % parts:
        raise ValueError(f"dimension {n} is not divisible by {parts}")
    step = n // parts
    return index * step, (index + 1) * step


def local_attention_shard(x: torch.Tensor, mesh: Mesh, rank: int) -> torch.Tensor:
    """This rank's block of a [B, H, N, D] tensor under P('dp', 'tp', None, None)."""
    d, t = mesh.coords(rank)
    b0, b1 = shard_bounds(x.shape[0], mesh.dp, d)
    h0, h1 = shard_bounds(x.shape[1], mesh.tp, t)
    return x[b0:b1, h0:h1]
