"""Training attention entry point — drop-in for the reference's
`pallas_flash.ops.interface.pallas_flash_attention`
(src/pallas_flash/ops/interface.py:20-85).

Same name and positional signature: `pallas_flash_attention(q, k, v)` takes
[B, H, N, D] tensors of any float dtype, casts them to bf16
(interface.py:23-25) and returns bf16 `o` shaped like q.  Keyword-only
additions (defaults keep the reference's behaviour): `causal`,
`sm_scale` (default 1/sqrt(D)), `return_lse`.  It is differentiable: the
backward pass (which the reference lacks) reuses the saved LSE.

Inputs may live on the GPU (the usual case) or on the host.  Host tensors are
copied to the current CUDA device (asynchronously when they are pinned) in
chunks of heads, pipelined with the kernels and with the copies back: `o`,
the LSE and, in the backward pass, dq / dk / dv come back as pinned host
tensors (one stream synchronisation per call).  Every compute step runs in
libpu_attn.so (sm_100a); there is no CPU fallback.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import _lib
from ..kernels.layout import kernel_head_dim, pad_head_dim

__all__ = ["pallas_flash_attention", "flash_attention_forward", "flash_attention_backward",
           "bwd_workspace_bytes"]


def _stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def flash_attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                            causal: bool = False, sm_scale: Optional[float] = None,
                            out: Optional[torch.Tensor] = None,
                            lse: Optional[torch.Tensor] = None):
    """Low-level forward on CUDA bf16 tensors with D in {64, 128}.

    Returns (o bf16 [B,H,Nq,D], lse fp32 [B,H,Nq]).  `out`/`lse` may be
    preallocated.  Calls pu_attn_fwd on the current stream.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(t, name)
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be bf16")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, H, Nq, D = q.shape
    Nkv = k.shape[2]
    if k.shape != (B, H, Nkv, D) or v.shape != k.shape:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((B, H, Nq), dtype=torch.float32, device=q.device)
    _lib.check(_lib.lib().pu_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                      lse.data_ptr(), B, H, Nq, Nkv, D, float(sm_scale),
                                      int(bool(causal)), _stream_handle()), "pu_attn_fwd")
    return out, lse


def bwd_workspace_bytes(B: int, H: int, Nq: int, D: int) -> int:
    return int(_lib.lib().pu_attn_bwd_workspace_size(B, H, Nq, D))


def flash_attention_backward(q, k, v, o, lse, do, *, causal: bool = False,
                             sm_scale: Optional[float] = None,
                             workspace: Optional[torch.Tensor] = None,
                             dq: Optional[torch.Tensor] = None,
                             dk: Optional[torch.Tensor] = None,
                             dv: Optional[torch.Tensor] = None,
                             deterministic: bool = False):
    """Low-level backward on CUDA bf16 tensors; returns (dq, dk, dv) bf16.

    `deterministic=True` selects pu_attn_bwd_deterministic (bitwise
    reproducible dQ, slower); the default pu_attn_bwd reduces dQ in fp32
    through L2, so its last bits may vary from run to run."""
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o), ("do", do)):
        _require_cuda(t, name)
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be bf16")
    q, k, v, o, do = (t.contiguous() for t in (q, k, v, o, do))
    lse = lse.contiguous()
    B, H, Nq, D = q.shape
    Nkv = k.shape[2]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    need = bwd_workspace_bytes(B, H, Nq, D)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    name = "pu_attn_bwd_deterministic" if deterministic else "pu_attn_bwd"
    _lib.check(getattr(_lib.lib(), name)(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                         lse.data_ptr(), do.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                         dv.data_ptr(), workspace.data_ptr(), need, B, H, Nq, Nkv, D,
                                         float(sm_scale), int(bool(causal)), _stream_handle()),
               name)
    return dq, dk, dv


class _FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, sm_scale):
        o, lse = flash_attention_forward(q, k, v, causal=causal, sm_scale=sm_scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal = causal
        ctx.sm_scale = sm_scale
        ctx.mark_non_differentiable(lse)
        return o, lse

    @staticmethod
    def backward(ctx, do, _dlse):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = flash_attention_backward(q, k, v, o, lse, do.to(torch.bfloat16),
                                              causal=ctx.causal, sm_scale=ctx.sm_scale)
        return dq, dk, dv, None, None


_HOST_CHUNKS = 8   # pipeline depth of the host path over the B*H heads


_COPY_STREAMS: dict = {}


def _copy_streams(dev: torch.device):
    """The (copy-in, copy-out) streams of `dev`, created once per device."""
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in _COPY_STREAMS:
        _COPY_STREAMS[key] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _COPY_STREAMS[key]


def _chunks(n: int, parts: int):
    """[a, b) row ranges splitting n rows into at most `parts` nearly equal parts."""
    parts = max(1, min(parts, n))
    return [(i * n // parts, (i + 1) * n // parts) for i in range(parts)]


def _h2d(dst: torch.Tensor, src: torch.Tensor, D: int, dev: torch.device):
    """Host rows `src` [n, N, D] into device rows `dst` [n, N, Dk] on the
    current stream: one copy straight into `dst` when Dk == D and `src` is a
    contiguous bf16 tensor, else through a device staging tensor (dtype cast,
    or the first D of Dk columns)."""
    if dst.shape[-1] == D and src.dtype == torch.bfloat16 and src.is_contiguous():
        dst.copy_(src, non_blocking=True)
    else:
        dst[..., :D].copy_(src.to(dev, non_blocking=True))


class _HostFlashAttention(torch.autograd.Function):
    """The attention of host tensors.  Heads are independent, so the B*H rows
    are processed in chunks on three streams: the host-to-device copy of chunk
    i+1, the kernels of chunk i and the device-to-host copy of chunk i-1 run
    at the same time (PCIe carries both directions at once).  Results land in
    pinned host tensors; the device copies of q, k, v, o and the LSE are kept
    for the backward pass.  Every head's kernels are the same as unchunked,
    so the results are identical."""

    @staticmethod
    def forward(ctx, q, k, v, causal, sm_scale, dev):
        B, H, Nq, D = q.shape
        Nkv = k.shape[2]
        Dk = kernel_head_dim(D)
        BH = B * H
        main = torch.cuda.current_stream(dev)
        s_in, s_out = _copy_streams(dev)
        hq, hk, hv = (t.detach().reshape(BH, t.shape[2], D) for t in (q, k, v))
        # unpadded head size: each chunk is copied straight into its slice
        # (no zero fill, no staging tensor); padded: zero-filled, then the
        # chunk lands in the first D columns
        alloc = torch.empty if Dk == D else torch.zeros
        q_ = alloc((BH, Nq, Dk), dtype=torch.bfloat16, device=dev)
        k_ = alloc((BH, Nkv, Dk), dtype=torch.bfloat16, device=dev)
        v_ = alloc((BH, Nkv, Dk), dtype=torch.bfloat16, device=dev)
        o = torch.empty((BH, Nq, Dk), dtype=torch.bfloat16, device=dev)
        lse = torch.empty((BH, Nq), dtype=torch.float32, device=dev)
        o_h = torch.empty((BH, Nq, D), dtype=torch.bfloat16, pin_memory=True)
        lse_h = torch.empty((BH, Nq), dtype=torch.float32, pin_memory=True)
        s_in.wait_stream(main)             # the zero fills above
        for a, b in _chunks(BH, _HOST_CHUNKS):
            with torch.cuda.stream(s_in):
                for h, d in ((hq, q_), (hk, k_), (hv, v_)):
                    _h2d(d[a:b], h[a:b], D, dev)
            main.wait_stream(s_in)
            flash_attention_forward(q_[a:b].unsqueeze(0), k_[a:b].unsqueeze(0), v_[a:b].unsqueeze(0),
                                    causal=causal, sm_scale=sm_scale, out=o[a:b].unsqueeze(0),
                                    lse=lse[a:b].unsqueeze(0))
            s_out.wait_stream(main)
            with torch.cuda.stream(s_out):
                o_h[a:b].copy_(o[a:b, :, :D], non_blocking=True)
                lse_h[a:b].copy_(lse[a:b], non_blocking=True)
        s_out.synchronize()
        ctx.save_for_backward(q_, k_, v_, o, lse)
        ctx.causal, ctx.sm_scale, ctx.dev, ctx.shape = causal, sm_scale, dev, (B, H, Nq, Nkv, D)
        lse_out = lse_h.view(B, H, Nq)
        ctx.mark_non_differentiable(lse_out)
        return o_h.view(B, H, Nq, D), lse_out

    @staticmethod
    def backward(ctx, do, _dlse):
        q_, k_, v_, o, lse = ctx.saved_tensors
        B, H, Nq, Nkv, D = ctx.shape
        BH, Dk, dev = B * H, q_.shape[-1], ctx.dev
        main = torch.cuda.current_stream(dev)
        s_in, s_out = _copy_streams(dev)
        hdo = do.detach().reshape(BH, Nq, D)
        do_ = (torch.empty if Dk == D else torch.zeros)((BH, Nq, Dk), dtype=torch.bfloat16, device=dev)
        dq = torch.empty((BH, Nq, Dk), dtype=torch.bfloat16, device=dev)
        dk = torch.empty((BH, Nkv, Dk), dtype=torch.bfloat16, device=dev)
        dv = torch.empty((BH, Nkv, Dk), dtype=torch.bfloat16, device=dev)
        parts = _chunks(BH, _HOST_CHUNKS)
        rows = max(b - a for a, b in parts)
        ws = torch.empty(bwd_workspace_bytes(1, rows, Nq, Dk), dtype=torch.uint8, device=dev)
        dq_h = torch.empty((BH, Nq, D), dtype=torch.bfloat16, pin_memory=True)
        dk_h = torch.empty((BH, Nkv, D), dtype=torch.bfloat16, pin_memory=True)
        dv_h = torch.empty((BH, Nkv, D), dtype=torch.bfloat16, pin_memory=True)
        s_in.wait_stream(main)
        for a, b in parts:
            with torch.cuda.stream(s_in):
                _h2d(do_[a:b], hdo[a:b], D, dev)
            main.wait_stream(s_in)
            c = lambda t: t[a:b].unsqueeze(0)   # noqa: E731
            flash_attention_backward(c(q_), c(k_), c(v_), c(o), c(lse), c(do_), causal=ctx.causal,
                                     sm_scale=ctx.sm_scale, workspace=ws, dq=c(dq), dk=c(dk), dv=c(dv))
            s_out.wait_stream(main)
            with torch.cuda.stream(s_out):
                for d, h in ((dq, dq_h), (dk, dk_h), (dv, dv_h)):
                    h[a:b].copy_(d[a:b, :, :D], non_blocking=True)
        s_out.synchronize()
        return (dq_h.view(B, H, Nq, D), dk_h.view(B, H, Nkv, D), dv_h.view(B, H, Nkv, D),
                None, None, None)


def pallas_flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                           causal: bool = False, sm_scale: Optional[float] = None,
                           return_lse: bool = False):
    """softmax(q k^T * sm_scale [+ causal mask]) v on the B200 kernels.

    q [B,H,Nq,D], k/v [B,H,Nkv,D] of any float dtype (cast to bf16, as the
    reference does).  Returns bf16 o shaped like q, or (o, lse) when
    `return_lse`.  Head sizes other than 64/128 are zero-padded for the
    kernel and sliced back (the reference's pad/unpad, layout.py); the scale
    defaults to 1/sqrt(D) of the true head size.
    """
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be [B, H, N, D]")
    D = q.shape[-1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if not q.is_cuda:
        dev = torch.device("cuda", torch.cuda.current_device())
        o, lse = _HostFlashAttention.apply(q, k, v, bool(causal), float(sm_scale), dev)
        return (o, lse) if return_lse else o
    q_, k_, v_ = (t.to(dtype=torch.bfloat16) for t in (q, k, v))
    Dk = kernel_head_dim(D)
    q_, k_, v_ = (pad_head_dim(t, Dk) for t in (q_, k_, v_))
    o, lse = _FlashAttention.apply(q_, k_, v_, bool(causal), float(sm_scale))
    if Dk != D:
        o = o[..., :D]
    return (o, lse) if return_lse else o
