"""Grouped K/V heads (GQA / MQA) and fp8 KV caches in the single-GPU decode
(pu_decode_gqa), against the oracle and against the MHA kernel on a cache
whose K/V heads are repeated.

  * G = H / H_kv from 2 to 64 with q and cache of one 16-bit type and
    D = 128: the tensor-core kernel (K tile x query slice, Vᵀ x Pᵀ; groups
    above 16 heads in slices of 16) against pu_decode on the repeated cache
    and the oracle; D = 64 with G = 16 runs the query-head kernel, whose
    split plan equals pu_decode's, so there the results match bit for bit
  * the CUDA-core grouped kernel (mixed q / cache dtypes, D = 64, G = 2, 4, 8)
  * fp16 / bf16 caches, ragged lengths (0, 1, partial chunks), D 64 / 128:
    vs the oracle (o max-abs 2e-2 / rel 1e-2, LSE 1e-3)
  * cache rows past a sequence's length holding NaN / Inf do not reach the
    output; scores that keep growing along the sequence (the running
    maximum moves many times, with rescales of the accumulated output)
  * fp8 (e4m3) caches with per-tensor scales: vs the oracle on the
    dequantised values (the same tolerance)
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import assert_close_lse, assert_close_o
from oracle import attention as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods(built_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from pallas_flash import _lib
    from pallas_flash.kernels import decoding
    _lib.device_status()
    return _lib, decoding


def _gen(shape, seed, dtype, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g) * scale).to(dtype)


def _f(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("H,H_kv,dt,D", [(16, 8, torch.float16, 128), (16, 4, torch.bfloat16, 128),
                                          (32, 4, torch.float16, 128), (64, 8, torch.bfloat16, 128),
                                          (24, 8, torch.float16, 128), (16, 1, torch.bfloat16, 128),
                                          (48, 2, torch.float16, 128), (32, 1, torch.float16, 128),
                                          (40, 1, torch.bfloat16, 128), (64, 1, torch.float16, 128),
                                          (16, 1, torch.bfloat16, 64)])
def test_gqa_equals_repeated_cache(mods, H, H_kv, dt, D):
    _lib, dec = mods
    B, N = 3, 3000
    q = _gen((B, H, 1, D), 1, dt)
    k = _gen((B, H_kv, N, D), 2, dt)
    v = _gen((B, H_kv, N, D), 3, dt)
    lens = torch.tensor([3000, 1, 1500], dtype=torch.int32, device="cuda")
    o, lse = dec.pallas_flash_decoding(q, k, v, kv_lens=lens, return_lse=True)
    G = H // H_kv
    kr, vr = k.repeat_interleave(G, dim=1), v.repeat_interleave(G, dim=1)
    o2, lse2 = dec.pallas_flash_decoding(q, kr, vr, kv_lens=lens, return_lse=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    if D == 128:
        assert_close_o(_f(o), _f(o2), max_abs=1e-2, rel=5e-3, what="grouped vs repeated cache")
        live = lens.cpu().numpy() > 0
        assert_close_lse(_f(lse)[live], _f(lse2)[live], tol=1e-4)
    else:
        assert torch.equal(o, o2) and torch.equal(lse, lse2)
    ro, rl = orc.decode_forward(_f(q), _f(k), _f(v), kv_lens=lens.cpu().numpy())
    assert_close_o(_f(o), ro, what=f"gqa H={H} H_kv={H_kv}")
    assert_close_lse(_f(lse), rl)


@pytest.mark.parametrize("D,H,H_kv,qdt", [(64, 8, 2, torch.bfloat16), (128, 32, 8, torch.bfloat16),
                                          (128, 32, 8, torch.float16)])
def test_gqa_vs_oracle(mods, D, H, H_kv, qdt):
    _lib, dec = mods
    B, N = 4, 2100
    q = _gen((B, H, 1, D), 10 + D, qdt)
    k = _gen((B, H_kv, N, D), 11 + D, torch.float16)
    v = _gen((B, H_kv, N, D), 12 + D, torch.float16)
    lens = torch.tensor([2100, 0, 257, 64], dtype=torch.int32, device="cuda")
    o, lse = dec.pallas_flash_decoding(q, k, v, kv_lens=lens, return_lse=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    ro, rl = orc.decode_forward(_f(q), _f(k), _f(v), kv_lens=lens.cpu().numpy())
    live = lens.cpu().numpy() > 0
    assert_close_o(_f(o), ro, what=f"gqa D={D}")
    assert_close_lse(_f(lse)[live], rl[live])
    assert (_f(o)[~live] == 0).all()


@pytest.mark.parametrize("H,H_kv", [(32, 32), (32, 8), (32, 4)])
def test_fp8_cache_vs_oracle(mods, H, H_kv):
    _lib, dec = mods
    fp8 = getattr(torch, "float8_e4m3fn", None)
    if fp8 is None:
        pytest.skip("torch without float8_e4m3fn")
    B, N, D = 2, 4096, 128
    q = _gen((B, H, 1, D), 20, torch.float16)
    k32 = _gen((B, H_kv, N, D), 21, torch.float32, 3.0)
    v32 = _gen((B, H_kv, N, D), 22, torch.float32, 2.0)
    k_scale, v_scale = 0.75, 0.5
    k8 = (k32 / k_scale).to(fp8)
    v8 = (v32 / v_scale).to(fp8)
    lens = torch.tensor([4096, 1000], dtype=torch.int32, device="cuda")
    o, lse = dec.pallas_flash_decoding(q, k8, v8, kv_lens=lens, return_lse=True,
                                       k_scale=k_scale, v_scale=v_scale)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    kd = _f(k8) * k_scale
    vd = _f(v8) * v_scale
    ro, rl = orc.decode_forward(_f(q), kd, vd, kv_lens=lens.cpu().numpy(), scale=1 / math.sqrt(D))
    assert_close_o(_f(o), ro, what="fp8 cache")
    assert_close_lse(_f(lse), rl)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gqa_stale_rows_past_length(mods, dt):
    """Rows past each sequence's length hold NaN and Inf (stale or never
    written cache slots): the output equals the oracle on the live rows."""
    _lib, dec = mods
    B, H, H_kv, N, D = 3, 32, 8, 1000, 128
    q = _gen((B, H, 1, D), 40, dt)
    k = _gen((B, H_kv, N, D), 41, dt)
    v = _gen((B, H_kv, N, D), 42, dt)
    lens = torch.tensor([1000, 130, 555], dtype=torch.int32, device="cuda")
    for b, n in enumerate(lens.tolist()):
        k[b, :, n:] = float("nan")
        v[b, :, n:] = float("inf")
    o, lse = dec.pallas_flash_decoding(q, k, v, kv_lens=lens, return_lse=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    assert torch.isfinite(o).all() and torch.isfinite(lse).all()
    kz, vz = k.clone(), v.clone()
    for b, n in enumerate(lens.tolist()):
        kz[b, :, n:] = 0
        vz[b, :, n:] = 0
    ro, rl = orc.decode_forward(_f(q), _f(kz), _f(vz), kv_lens=lens.cpu().numpy())
    assert_close_o(_f(o), ro, what="stale rows")
    assert_close_lse(_f(lse), rl)


def test_gqa_growing_scores(mods):
    """K rows scaled up along the sequence, so each tile's scores exceed the
    running maximum of the previous ones and the output accumulated so far is
    rescaled again and again; per head the growth differs."""
    _lib, dec = mods
    B, H, H_kv, N, D = 2, 16, 4, 4096, 128
    dt = torch.float16
    q = _gen((B, H, 1, D), 50, dt)
    ramp = torch.linspace(0.2, 4.0, N, device="cuda").view(1, 1, N, 1)
    k = (_gen((B, H_kv, N, D), 51, torch.float32) * 0.3 + 0.5 * q.float().view(B, H_kv, H // H_kv, D)[:, :, :1, :]) * ramp
    k = k.to(dt)
    v = _gen((B, H_kv, N, D), 52, dt)
    o, lse = dec.pallas_flash_decoding(q, k, v, return_lse=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    ro, rl = orc.decode_forward(_f(q), _f(k), _f(v))
    assert_close_o(_f(o), ro, what="growing scores")
    assert_close_lse(_f(lse), rl)


@pytest.mark.parametrize("H,H_kv", [(32, 8), (16, 16)])
def test_fp8_cache_every_code(mods, H, H_kv):
    """Every finite e4m3 code, subnormals and the largest magnitudes included,
    appears in K and V; the kernel decodes them exactly (the oracle sees the
    same dequantised values).  Scores stay small so all rows matter."""
    _lib, dec = mods
    fp8 = getattr(torch, "float8_e4m3fn", None)
    if fp8 is None:
        pytest.skip("torch without float8_e4m3fn")
    B, N, D = 1, 2032, 128
    codes = torch.tensor([c for c in range(256) if c not in (0x7F, 0xFF)], dtype=torch.uint8)
    idx = (torch.arange(N)[:, None] * 7 + torch.arange(D)[None, :] * 3) % codes.numel()
    k8 = codes[idx].view(fp8).expand(B, H_kv, N, D).contiguous().cuda()
    v8 = codes[(idx + 101) % codes.numel()].view(fp8).expand(B, H_kv, N, D).contiguous().cuda()
    q = _gen((B, H, 1, D), 23, torch.float16, 0.02)
    k_scale, v_scale = 1.0 / 448.0, 1.0 / 32.0
    o, lse = dec.pallas_flash_decoding(q, k8, v8, return_lse=True, k_scale=k_scale, v_scale=v_scale)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    kd = _f(k8) * k_scale
    vd = _f(v8) * v_scale
    ro, rl = orc.decode_forward(_f(q), kd, vd, scale=1 / math.sqrt(D))
    assert_close_o(_f(o), ro, what="fp8 every code")
    assert_close_lse(_f(lse), rl)
