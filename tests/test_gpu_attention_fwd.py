"""GPU parity of the tcgen05 attention forward (pu_attn_fwd) against the oracle.

Cases follow the reference's tests: tests/test_correctness.py:35-74 (five
shapes, inputs N(0,1)*0.5, aligned and unaligned N and D) and
tests/test_numerics.py:29-117 (known answers at B,H,N,D = 2,2,512,128),
plus causal variants, LSE, ragged lengths and the c1 benchmark shape.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import assert_close_lse, assert_close_o, randn, to_np
from oracle import attention as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pf(built_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from pallas_flash.ops import interface
    return interface


def _check(pf, B, H, Nq, Nkv, D, causal, seed, scale=1.0):
    q = randn((B, H, Nq, D), seed, scale)
    k = randn((B, H, Nkv, D), seed + 1, scale)
    v = randn((B, H, Nkv, D), seed + 2, scale)
    o, lse = pf.pallas_flash_attention(q.cuda(), k.cuda(), v.cuda(), causal=causal,
                                       return_lse=True)
    torch.cuda.synchronize()
    from pallas_flash import _lib
    assert _lib.device_status()[0] == 0
    assert o.dtype == torch.bfloat16 and o.shape == q.shape
    ro, rl = orc.mha_forward(to_np(q), to_np(k), to_np(v), causal=causal,
                             scale=1.0 / math.sqrt(D))
    assert_close_o(to_np(o), ro)
    assert_close_lse(to_np(lse), rl)
    return o


@pytest.mark.parametrize("B,H,N,D", [(1, 2, 1024, 64), (2, 2, 1500, 128), (2, 2, 1000, 100),
                                     (2, 4, 1024, 128), (1, 2, 2048, 128)])
def test_reference_correctness_shapes(pf, B, H, N, D):
    """tests/test_correctness.py shapes, non-causal, N(0,1)*0.5 inputs."""
    _check(pf, B, H, N, N, D, causal=False, seed=42, scale=0.5)


@pytest.mark.parametrize("B,H,N,D", [(1, 2, 1024, 64), (2, 2, 1500, 128), (1, 3, 384, 128),
                                     (1, 4, 1024, 128)])
def test_causal(pf, B, H, N, D):
    _check(pf, B, H, N, N, D, causal=True, seed=7)


@pytest.mark.parametrize("Nq,Nkv,causal", [(1, 1, False), (7, 7, True), (129, 129, True),
                                           (128, 1000, False), (300, 77, False), (256, 640, True)])
def test_ragged_lengths(pf, Nq, Nkv, causal):
    _check(pf, 1, 2, Nq, Nkv, 128, causal=causal, seed=11)


def test_c1_benchmark_shape(pf):
    """Causal B=1 H=4 N=1024 D=128, N(0,1) inputs, scale 1/sqrt(128)."""
    _check(pf, 1, 4, 1024, 1024, 128, causal=True, seed=0)


def test_kernel_emulation_agrees(pf):
    """The reference kernel's own arithmetic (bf16 P, 128-blocks) agrees too."""
    q = randn((1, 2, 512, 128), 5)
    k = randn((1, 2, 512, 128), 6)
    v = randn((1, 2, 512, 128), 7)
    o = pf.pallas_flash_attention(q.cuda(), k.cuda(), v.cuda())
    eo, _, _ = orc.pipeline_emulation(to_np(q), to_np(k), to_np(v))
    assert_close_o(to_np(o), eo)


B, H, N, D = 2, 2, 512, 128


def test_numerics_extreme_magnitude(pf):
    """test_numerics.py:29-61: q = k = 100, v = 1 -> output is exactly 1."""
    q = torch.full((B, H, N, D), 100.0, dtype=torch.bfloat16, device="cuda")
    v = torch.ones((B, H, N, D), dtype=torch.bfloat16, device="cuda")
    out = pf.pallas_flash_attention(q, q, v)
    assert torch.isfinite(out.float()).all()
    np.testing.assert_allclose(to_np(out), np.ones((B, H, N, D)), atol=1e-2)


def test_numerics_zero_variance(pf):
    """test_numerics.py:63-80: q = k = 0 -> finite (uniform average of v)."""
    q = torch.zeros((B, H, N, D), dtype=torch.bfloat16, device="cuda")
    v = randn((B, H, N, D), 0).cuda()
    out = pf.pallas_flash_attention(q, q, v)
    assert torch.isfinite(out.float()).all()
    expect = to_np(v).mean(axis=2, keepdims=True).repeat(N, axis=2)
    assert_close_o(to_np(out), expect)


def test_numerics_highly_negative_keys(pf):
    """test_numerics.py:82-99: k = -1e4 -> finite output."""
    q = randn((B, H, N, D), 1).cuda()
    k = torch.full((B, H, N, D), -1e4, dtype=torch.bfloat16, device="cuda")
    v = randn((B, H, N, D), 2).cuda()
    out = pf.pallas_flash_attention(q, k, v)
    assert torch.isfinite(out.float()).all()


def test_numerics_precision_preservation(pf):
    """test_numerics.py:101-117: output dtype is bf16 even for fp32 inputs."""
    q = randn((B, H, N, D), 3, dtype=torch.float32).cuda()
    out = pf.pallas_flash_attention(q, q, q)
    assert out.dtype == torch.bfloat16


def test_host_tensors_roundtrip(pf):
    """CPU inputs are copied to the GPU and the result comes back to the host."""
    q = randn((1, 2, 256, 128), 9)
    out = pf.pallas_flash_attention(q, q, q, causal=True)
    assert out.device.type == "cpu"
    ro, _ = orc.mha_forward(to_np(q), to_np(q), to_np(q), causal=True)
    assert_close_o(to_np(out), ro)


@pytest.mark.parametrize("D", [128, 80])
def test_host_tensors_backward(pf, D):
    """Host inputs with gradients: o and dq / dk / dv come back as pinned host
    tensors equal to the ones the device path computes (same kernels)."""
    shape = (1, 2, 384, D)
    q, k, v = (randn(shape, 20 + i).requires_grad_() for i in range(3))
    do = randn(shape, 30).pin_memory()
    o = pf.pallas_flash_attention(q, k, v, causal=True)
    assert o.device.type == "cpu" and o.is_pinned() and o.dtype == torch.bfloat16
    o.backward(do)
    assert all(t.grad is not None and t.grad.device.type == "cpu" for t in (q, k, v))
    qd, kd, vd = (t.detach().cuda().requires_grad_() for t in (q, k, v))
    od = pf.pallas_flash_attention(qd, kd, vd, causal=True)
    od.backward(do.cuda())
    assert torch.equal(o, od.cpu())
    for h, d in ((q, qd), (k, kd), (v, vd)):
        assert torch.equal(h.grad, d.grad.cpu())
