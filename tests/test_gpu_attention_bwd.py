"""GPU parity of the tcgen05 attention backward (pu_attn_bwd) against the
oracle's closed-form gradients of the reference's attention
(benchmarks/baseline_mha.py:22-58; the reference has no backward kernel).
Bar: dQ, dK, dV within 3e-2 norm-relative error."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import assert_close_grad, randn, to_np
from oracle import attention as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pf(built_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from pallas_flash.ops import interface
    return interface


def _grads(pf, B, H, Nq, Nkv, D, causal, seed, scale=1.0, deterministic=False):
    q = randn((B, H, Nq, D), seed, scale)
    k = randn((B, H, Nkv, D), seed + 1, scale)
    v = randn((B, H, Nkv, D), seed + 2, scale)
    do = randn((B, H, Nq, D), seed + 3)
    qc, kc, vc, dc = (t.cuda() for t in (q, k, v, do))
    o, lse = pf.flash_attention_forward(qc, kc, vc, causal=causal)
    dq, dk, dv = pf.flash_attention_backward(qc, kc, vc, o, lse, dc, causal=causal,
                                             deterministic=deterministic)
    torch.cuda.synchronize()
    from pallas_flash import _lib
    assert _lib.device_status()[0] == 0
    sc = 1.0 / math.sqrt(D)
    ro, rl = orc.mha_forward(to_np(q), to_np(k), to_np(v), causal=causal, scale=sc)
    rdq, rdk, rdv = orc.mha_backward(to_np(q), to_np(k), to_np(v), ro, rl, to_np(do),
                                     causal=causal, scale=sc)
    assert_close_grad(to_np(dq), rdq, what="dq")
    assert_close_grad(to_np(dk), rdk, what="dk")
    assert_close_grad(to_np(dv), rdv, what="dv")
    return dq, dk, dv


@pytest.mark.parametrize("B,H,N,D,causal", [(1, 2, 256, 128, False), (1, 2, 256, 128, True),
                                            (2, 2, 1024, 128, True), (1, 2, 1024, 64, True),
                                            (1, 2, 1500, 128, False), (2, 3, 640, 64, False),
                                            (1, 9, 384, 128, True)])
@pytest.mark.parametrize("deterministic", [False, True], ids=["fused", "deterministic"])
def test_backward_matches_oracle(pf, B, H, N, D, causal, deterministic):
    _grads(pf, B, H, N, N, D, causal, seed=21, deterministic=deterministic)


@pytest.mark.parametrize("Nq,Nkv,causal", [(1, 1, False), (77, 77, True), (129, 300, False),
                                           (300, 129, False), (200, 333, True), (129, 1, False)])
@pytest.mark.parametrize("deterministic", [False, True], ids=["fused", "deterministic"])
def test_backward_ragged(pf, Nq, Nkv, causal, deterministic):
    _grads(pf, 1, 2, Nq, Nkv, 128, causal, seed=31, deterministic=deterministic)


def test_autograd_path(pf):
    """pallas_flash_attention is differentiable through torch.autograd."""
    from pallas_flash.ops.interface import pallas_flash_attention
    q = randn((1, 2, 384, 128), 41).cuda().requires_grad_(True)
    k = randn((1, 2, 384, 128), 42).cuda().requires_grad_(True)
    v = randn((1, 2, 384, 128), 43).cuda().requires_grad_(True)
    do = randn((1, 2, 384, 128), 44).cuda()
    o = pallas_flash_attention(q, k, v, causal=True)
    o.backward(do)
    ro, rl = orc.mha_forward(to_np(q), to_np(k), to_np(v), causal=True)
    rdq, rdk, rdv = orc.mha_backward(to_np(q), to_np(k), to_np(v), ro, rl, to_np(do), causal=True)
    assert_close_grad(to_np(q.grad), rdq, what="dq")
    assert_close_grad(to_np(k.grad), rdk, what="dk")
    assert_close_grad(to_np(v.grad), rdv, what="dv")


def test_backward_deterministic_dk_dv(pf):
    """dK and dV are reduced inside one CTA on both paths: bitwise identical
    across runs; the deterministic path's dQ is bitwise identical too, and the
    fused path's dQ (fp32 reductions in L2) differs only in its last bits."""
    q = randn((1, 4, 512, 128), 51).cuda()
    k = randn((1, 4, 512, 128), 52).cuda()
    v = randn((1, 4, 512, 128), 53).cuda()
    do = randn((1, 4, 512, 128), 54).cuda()
    o, lse = pf.flash_attention_forward(q, k, v, causal=True)
    a = pf.flash_attention_backward(q, k, v, o, lse, do, causal=True)
    b = pf.flash_attention_backward(q, k, v, o, lse, do, causal=True)
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])
    assert (a[0].float() - b[0].float()).abs().max().item() < 1e-2
    c = pf.flash_attention_backward(q, k, v, o, lse, do, causal=True, deterministic=True)
    d = pf.flash_attention_backward(q, k, v, o, lse, do, causal=True, deterministic=True)
    assert all(torch.equal(x, y) for x, y in zip(c, d))
    # both paths round the same P and dS to bf16: dK and dV agree bitwise
    assert torch.equal(a[1], c[1]) and torch.equal(a[2], c[2])
    assert (a[0].float() - c[0].float()).abs().max().item() < 1e-2


def test_fused_matches_deterministic_large(pf):
    """The fused and the two-kernel backward agree on a causal B1 H4 N4096
    case (many key tiles add into each dQ row)."""
    q = randn((1, 4, 4096, 128), 61).cuda()
    k = randn((1, 4, 4096, 128), 62).cuda()
    v = randn((1, 4, 4096, 128), 63).cuda()
    do = randn((1, 4, 4096, 128), 64).cuda()
    o, lse = pf.flash_attention_forward(q, k, v, causal=True)
    a = pf.flash_attention_backward(q, k, v, o, lse, do, causal=True)
    c = pf.flash_attention_backward(q, k, v, o, lse, do, causal=True, deterministic=True)
    from pallas_flash import _lib
    assert _lib.device_status()[0] == 0
    assert torch.equal(a[1], c[1]) and torch.equal(a[2], c[2])
    r = orc.compare(to_np(a[0]), to_np(c[0]))
    assert r["rel"] <= 5e-3, r
