"""Padding helpers (mirror of the reference's src/pallas_flash/kernels/layout.py).

The reference pads N and D to multiples of 128 before every pallas_call
(layout.py:41-82) and slices the result back (layout.py:84-103).  The B200
kernels take any sequence length directly (TMA zero-fills out-of-range rows
and the kernels mask keys past N), so only head sizes other than 64/128 are
padded here — the tensor-map row pitch must be a multiple of 16 bytes.
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch

MXU_SIZE = 128  # the reference's alignment unit (config.py:64)


def get_padded_dim(dim: int, alignment: int = MXU_SIZE) -> int:
    """Smallest multiple of `alignment` >= dim (layout.py:28-39)."""
    return (dim + alignment - 1) // alignment * alignment


def pad_tensor(x: torch.Tensor, axes: Sequence[int] = (-2, -1),
               alignment: int = MXU_SIZE) -> Tuple[torch.Tensor, Tuple[int, ...]]:
    """Zero-pad the given axes to multiples of `alignment` (layout.py:41-82)."""
    original_shape = tuple(x.shape)
    rank = x.dim()
    norm = {a % rank for a in axes}
    pads = []
    need = False
    for i in reversed(range(rank)):
        amount = get_padded_dim(x.shape[i], alignment) - x.shape[i] if i in norm else 0
        need = need or amount > 0
        pads += [0, amount]
    if not need:
        return x, original_shape
    return torch.nn.functional.pad(x, pads), original_shape


def unpad_tensor(x: torch.Tensor, original_shape: Tuple[int, ...]) -> torch.Tensor:
    """Slice back to `original_shape` (layout.py:84-103)."""
    if tuple(x.shape) == tuple(original_shape):
        return x
    return x[tuple(slice(0, d) for d in original_shape)]


def kernel_head_dim(d: int) -> int:
    """Head size the kernels run at: 64 or 128 (others are zero-padded)."""
    if d <= 64:
        return 64
    if d <= 128:
        return 128
    raise ValueError(f"head size {d} is above 128, which the kernels do not support")


def pad_head_dim(x: torch.Tensor, d_kernel: int) -> torch.Tensor:
    if x.shape[-1] == d_kernel:
        return x
    return torch.nn.functional.pad(x, (0, d_kernel - x.shape[-1]))
