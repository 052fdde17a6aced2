"""Output projection fused with the TP all-reduce (pu_outproj_allreduce) on
one GPU (a one-rank group): the tcgen05 GEMM and the reduce / receive path
against an fp32 product, over consecutive calls (both exchange slots), and
the bounded wait of the reduction.  T a multiple of 256 runs the CTA-pair
kernel (cta_group::2, 256 x 256 tiles), other T the single-CTA kernel; both
are checked against the fp32 product and against each other on the same
inputs.  The two-GPU exchange is covered in test_gpu_multigpu.py.

Tolerance: the result is the bf16 rounding of an fp32-accumulated product,
so max |y - ref| <= 1e-2 * max |ref| and ||y - ref|| / ||ref|| <= 5e-3.
"""
from __future__ import annotations

import ctypes
import datetime

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def group(built_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import torch.distributed as dist
    from helpers import one_rank_init_method
    already = dist.is_initialized()
    if not already:
        dist.init_process_group("gloo", init_method=one_rank_init_method(), rank=0,
                                world_size=1, timeout=datetime.timedelta(seconds=30))
    yield dist.group.WORLD
    from pallas_flash.distributed import peer
    peer.close_all()
    if not already:
        dist.destroy_process_group()


def _gen(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


def _check(y, ref):
    err = (y.float() - ref).abs().max().item()
    rel = ((y.float() - ref).norm() / ref.norm()).item()
    assert err <= 1e-2 * ref.abs().max().item() and rel <= 5e-3, (err, rel)


@pytest.mark.parametrize("T,K,N", [(128, 64, 256), (640, 192, 768), (2048, 2048, 2048), (256, 64, 256),
                                   (512, 192, 768), (1280, 1024, 512), (4096, 128, 2048)])
def test_outproj_one_rank(group, T, K, N):
    from pallas_flash import _lib
    from pallas_flash.distributed.outproj import out_proj_all_reduce
    for step in range(3):
        o = _gen((T, K), 10 * step + 1)
        w = _gen((K, N), 10 * step + 2, 1.0 / K ** 0.5)
        y = out_proj_all_reduce(o, w, group)
        torch.cuda.synchronize()
        _check(y, o.float() @ w.float())
    assert _lib.device_status() == (0, 0)


@pytest.mark.parametrize("T,K,N", [(256, 64, 256), (768, 576, 1280), (16384, 2048, 2048)])
def test_outproj_pair_matches_single(group, T, K, N, monkeypatch):
    """The CTA-pair kernel against the single-CTA kernel on the same inputs:
    both accumulate each output in fp32 over the same K steps of 16, so the
    results agree to the last bf16 bit or nearly (|diff| <= 1 ulp of bf16
    on at most 0.1 % of the outputs)."""
    from pallas_flash import _lib
    from pallas_flash.distributed.outproj import out_proj_all_reduce
    o = _gen((T, K), 71)
    w = _gen((K, N), 72, 1.0 / K ** 0.5)
    y_pair = out_proj_all_reduce(o, w, group)
    monkeypatch.setenv("PU_OUTPROJ_PAIR", "0")
    y_single = out_proj_all_reduce(o, w, group)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    d = (y_pair.float() - y_single.float()).abs()
    ulp = y_single.float().abs().clamp_min(1e-30) * 2.0 ** -7
    assert (d <= ulp).all(), d.max().item()
    assert (d > 0).float().mean().item() <= 1e-3
    if T * N <= (1 << 21):
        _check(y_pair, o.float() @ w.float())


def test_outproj_wait_runs_out(group):
    """A two-rank layout whose second rank never publishes (both buffers are
    this GPU's own): the reduction and the receive give up after their limit
    and report PU_ERR_DEVICE_TIMEOUT / 401; the next call works."""
    from pallas_flash import _lib
    from pallas_flash.distributed.outproj import out_proj_all_reduce
    lib = _lib.lib()
    T, K, N = 128, 64, 512
    nbytes = int(lib.pu_outproj_exchange_bytes(T, N, 2))
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    ptrs = (ctypes.c_void_p * 2)(*[b.data_ptr() for b in bufs])
    o = _gen((T, K), 3)
    w = _gen((K, N), 4)
    y = torch.zeros((T, N), dtype=torch.bfloat16, device="cuda")
    _lib.check(lib.pu_outproj_allreduce(o.data_ptr(), w.data_ptr(), y.data_ptr(), ptrs, 2, 0, 1,
                                        T, K, N, 20_000_000, torch.cuda.current_stream().cuda_stream),
               "pu_outproj_allreduce")
    assert _lib.device_status() == (_lib.PU_ERR_DEVICE_TIMEOUT, 401)
    y2 = out_proj_all_reduce(o, w, group)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    _check(y2, o.float() @ w.float())


def test_outproj_argument_errors(group):
    from pallas_flash import _lib
    lib = _lib.lib()
    d = 1 << 12
    ptrs = (ctypes.c_void_p * 1)(d)
    assert lib.pu_outproj_allreduce(d, d, d, ptrs, 1, 0, 1, 100, 64, 256, 1000, None) == _lib.PU_ERR_UNSUPPORTED
    assert lib.pu_outproj_allreduce(d, d, d, ptrs, 1, 0, 0, 128, 64, 256, 1000, None) == _lib.PU_ERR_INVALID_ARGUMENT
    assert lib.pu_outproj_exchange_bytes(128, 200, 1) == 0
