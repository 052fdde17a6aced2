"""Attention output projection with the tensor-parallel all-reduce.

The reference's TP scheme (src/pallas_flash/distributed/collectives.py:27-41)
runs each device's attention heads independently, multiplies by the matching
rows of W_O, and sums the partial projections with `all_reduce_tp` (a psum
over the 'tp' axis).  `out_proj_all_reduce` is that step:

  transport="peer"  one call of pu_outproj_allreduce: a tcgen05 GEMM whose
                    epilogue stores each bf16 partial tile into its owner
                    rank's buffer over NVLink, owner reduce + broadcast, and a
                    copy into the result (no NCCL call)
  transport="nccl"  torch matmul (cuBLAS) + an NCCL all-reduce of the bf16
                    partial product, the unfused path, for comparison

Every rank passes its o_local [T, K] and w_local [K, N] (bf16) and receives
y [T, N] = sum over ranks of o_local @ w_local.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _lib
from .peer import PeerBuffers, get_cached

__all__ = ["out_proj_all_reduce", "OutProjExchange"]

DEFAULT_TIMEOUT_NS = 1_000_000_000


class OutProjExchange(PeerBuffers):
    """Peer buffers for one (T, N) output shape."""

    def __init__(self, T: int, N: int, group=None):
        g = group if group is not None else dist.group.WORLD
        G = dist.get_world_size(g)
        nbytes = int(_lib.lib().pu_outproj_exchange_bytes(T, N, G))
        if nbytes == 0:
            raise ValueError(f"T={T} must be a multiple of 128 and N={N} of 256")
        self.T, self.N = T, N
        super().__init__(nbytes, g)

    def all_reduce(self, o_local: torch.Tensor, w_local: torch.Tensor, out: torch.Tensor,
                   timeout_ns: int = DEFAULT_TIMEOUT_NS) -> torch.Tensor:
        T, K = o_local.shape
        N = w_local.shape[1]
        epoch = self.next_epoch()
        _lib.check(_lib.lib().pu_outproj_allreduce(
            o_local.data_ptr(), w_local.data_ptr(), out.data_ptr(), self._ptrs, self.world,
            self.rank, epoch, T, K, N, int(timeout_ns), torch.cuda.current_stream().cuda_stream),
            "pu_outproj_allreduce")
        return out


def out_proj_all_reduce(o_local: torch.Tensor, w_local: torch.Tensor, group=None, *,
                        transport: str = "peer", out=None,
                        timeout_ns: int = DEFAULT_TIMEOUT_NS) -> torch.Tensor:
    """y = sum over the ranks of `group` of o_local @ w_local, on every rank (bf16)."""
    if o_local.dim() != 2 or w_local.dim() != 2 or o_local.shape[1] != w_local.shape[0]:
        raise ValueError(f"shapes {tuple(o_local.shape)} x {tuple(w_local.shape)}")
    o_local = o_local.to(torch.bfloat16).contiguous()
    w_local = w_local.to(torch.bfloat16).contiguous()
    T, N = o_local.shape[0], w_local.shape[1]
    if out is None:
        out = torch.empty((T, N), dtype=torch.bfloat16, device=o_local.device)
    if transport == "nccl":
        torch.matmul(o_local, w_local, out=out)
        dist.all_reduce(out, group=group)
        return out
    if transport != "peer":
        raise ValueError(f"unknown transport {transport!r} (peer or nccl)")
    ex = get_cached(("outproj", T, N), lambda: OutProjExchange(T, N, group), group)
    return ex.all_reduce(o_local, w_local, out, timeout_ns)
