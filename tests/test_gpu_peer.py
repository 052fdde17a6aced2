"""Peer-memory decode exchange on one GPU (a one-rank group): the push/pull
kernels against the NCCL-path kernels (pu_decode_partial + pu_decode_combine)
and the bounded wait of the pull.  The two-GPU exchange is covered in
test_gpu_multigpu.py."""
from __future__ import annotations

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


def _gen(shape, seed, dtype=torch.float16):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, device="cuda", generator=g).to(dtype)


def test_push_pull_equals_partial_combine(group):
    from pallas_flash import _lib
    from pallas_flash.kernels import decoding as dec
    B, H, N, D = 3, 8, 5000, 128
    k = _gen((B, H, N, D), 1)
    v = _gen((B, H, N, D), 2)
    lens = torch.tensor([5000, 17, 0], dtype=torch.int32, device="cuda")
    for step in range(4):   # both exchange slots, twice
        q = _gen((B, H, 1, D), 10 + step)
        part = dec.decode_partial(q, k, v, kv_offset=0, kv_lens=lens)
        o_ref, l_ref = dec.decode_combine(part[None], B, H, D)
        o, l = dec.pallas_flash_decoding(q, k, v, kv_lens=lens, group=group, transport="peer",
                                         return_lse=True)
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref) and torch.equal(l, l_ref), step
    assert _lib.device_status() == (0, 0)


def test_unfused_merge_for_large_batches(group):
    """B*H above half the CTA slots: the merge runs as a second kernel."""
    from pallas_flash import _lib
    from pallas_flash.kernels import decoding as dec
    B, H, N, D = 5, 32, 600, 64
    k = _gen((B, H, N, D), 21)
    v = _gen((B, H, N, D), 22)
    for step in range(3):
        q = _gen((B, H, 1, D), 30 + step)
        part = dec.decode_partial(q, k, v, kv_offset=0)
        o_ref, l_ref = dec.decode_combine(part[None], B, H, D)
        o, l = dec.pallas_flash_decoding(q, k, v, group=group, transport="peer", return_lse=True)
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref) and torch.equal(l, l_ref), step
    assert _lib.device_status() == (0, 0)


def test_pull_wait_runs_out(group):
    """A merge for an epoch nobody publishes gives up after its limit,
    reports PU_ERR_DEVICE_TIMEOUT / 304, and later steps still work."""
    from pallas_flash import _lib
    from pallas_flash.distributed import peer
    from pallas_flash.kernels import decoding as dec
    B, H, N, D = 1, 4, 1024, 64
    k = _gen((B, H, N, D), 3, torch.bfloat16)
    v = _gen((B, H, N, D), 4, torch.bfloat16)
    q = _gen((B, H, 1, D), 5, torch.bfloat16)
    dec.pallas_flash_decoding(q, k, v, group=group, transport="peer")
    ex = peer.get_exchange(B, H, D, group)
    o = torch.full((B, H, 1, D), 7.0, dtype=torch.bfloat16, device="cuda")
    _lib.check(_lib.lib().pu_decode_pull(ex._local, 1, ex.epoch + 10, o.data_ptr(), None, B, H, D,
                                         20_000_000, torch.cuda.current_stream().cuda_stream),
               "pu_decode_pull")
    assert _lib.device_status() == (_lib.PU_ERR_DEVICE_TIMEOUT, 304)
    assert (o == 0).all()
    o2 = dec.pallas_flash_decoding(q, k, v, group=group, transport="peer")
    ref = dec.pallas_flash_decoding(q, k, v)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    assert (o2.float() - ref.float()).abs().max().item() < 1e-2


def test_push_argument_errors(group):
    from pallas_flash import _lib
    lib = _lib.lib()
    rc = lib.pu_decode_pull(1 << 12, 9, 1, 1 << 12, None, 1, 1, 128, 1000, None)
    assert rc == _lib.PU_ERR_UNSUPPORTED
    rc = lib.pu_decode_pull(1 << 12, 2, 0, 1 << 12, None, 1, 1, 128, 1000, None)
    assert rc == _lib.PU_ERR_INVALID_ARGUMENT
    rc = lib.pu_decode_pull(1 << 12, 2, 1, 1 << 12, None, 1, 1, 128, 3_000_000_000, None)
    assert rc == _lib.PU_ERR_INVALID_ARGUMENT
