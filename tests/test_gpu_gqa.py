"""Grouped K/V heads (GQA / MQA) and fp8 KV caches in the single-GPU decode
(pu_decode_gqa), against the oracle and against the MHA kernel on a cache
whose K/V heads are repeated.

  * H_kv in {H/2, H/4, H/8}: the grouped kernel (one CTA per K/V head for
    all its query heads) against pu_decode on the repeated cache and the
    oracle; H_kv = 1 with 16 query heads runs the query-head kernel, whose
    split plan equals pu_decode's, so there the results match bit for bit
  * fp16 / bf16 caches, ragged lengths (0, 1, partial chunks), D 64 / 128:
    vs the oracle (o max-abs 2e-2 / rel 1e-2, LSE 1e-3)
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


@pytest.mark.parametrize("H,H_kv,dt", [(16, 8, torch.float16), (16, 4, torch.bfloat16),
                                        (32, 4, torch.float16), (64, 8, torch.bfloat16),
                                        (16, 1, torch.bfloat16)])
def test_gqa_equals_repeated_cache(mods, H, H_kv, dt):
    _lib, dec = mods
    B, N, D = 3, 3000, 128
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
    if G in (2, 4, 8):
        assert_close_o(_f(o), _f(o2), max_abs=1e-2, rel=5e-3, what="grouped vs repeated cache")
        live = lens.cpu().numpy() > 0
        assert_close_lse(_f(lse)[live], _f(lse2)[live], tol=1e-4)
    else:
        assert torch.equal(o, o2) and torch.equal(lse, lse2)
    ro, rl = orc.decode_forward(_f(q), _f(k), _f(v), kv_lens=lens.cpu().numpy())
    assert_close_o(_f(o), ro, what=f"gqa H={H} H_kv={H_kv}")
    assert_close_lse(_f(lse), rl)


@pytest.mark.parametrize("D,H,H_kv", [(64, 8, 2), (128, 32, 8)])
def test_gqa_vs_oracle(mods, D, H, H_kv):
    _lib, dec = mods
    B, N = 4, 2100
    q = _gen((B, H, 1, D), 10 + D, torch.bfloat16)
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
