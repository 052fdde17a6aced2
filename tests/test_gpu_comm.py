"""The library's own NCCL communicator (pu_comm_unique_id / pu_comm_init /
pu_allgather_partials / pu_comm_destroy) on one GPU: a one-rank all-gather
returns the partial unchanged, and the sequence-sharded decode with
transport="lib" matches the oracle (o max-abs 2e-2 / rel 1e-2, LSE 1e-3).
The two-rank exchange (bit-identical to the torch.distributed route) is in
test_gpu_multigpu.py."""
from __future__ import annotations

import datetime

import pytest
import torch

from helpers import randn
from oracle import attention as orc

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
    from pallas_flash.distributed.collectives import close_lib_comms
    close_lib_comms()
    if not already:
        dist.destroy_process_group()


def test_one_rank_all_gather_is_identity(group):
    from pallas_flash.distributed.collectives import LibComm
    B, H, D = 3, 8, 128
    comm = LibComm(group)
    for seed in (1, 2):
        part = randn((B * H, D + 2), seed, dtype=torch.float32).cuda()
        out = comm.all_gather(part, B, H, D)
        torch.cuda.synchronize()
        assert out.shape == (1, B * H, D + 2) and torch.equal(out[0], part)
    with pytest.raises(TypeError):
        comm.all_gather(part.to(torch.bfloat16), B, H, D)
    comm.close()


def test_sharded_decode_lib_transport(group):
    from pallas_flash import _lib
    from pallas_flash.kernels.decoding import pallas_flash_decoding
    B, H, N, D = 2, 8, 3000, 128
    q = randn((B, H, 1, D), 11, dtype=torch.float16)
    k = randn((B, H, N, D), 12, dtype=torch.float16)
    v = randn((B, H, N, D), 13, dtype=torch.float16)
    lens = torch.tensor([3000, 1200], dtype=torch.int32)
    o, lse = pallas_flash_decoding(q.cuda(), k.cuda(), v.cuda(), kv_lens=lens.cuda(), group=group,
                                   transport="lib", return_lse=True)
    torch.cuda.synchronize()
    assert _lib.device_status() == (0, 0)
    ro, rl = orc.decode_forward(q.float().numpy(), k.float().numpy(), v.float().numpy(), kv_lens=lens.numpy())
    c = orc.compare(o.float().cpu().numpy(), ro)
    assert c["max_abs"] <= 2e-2 and c["rel"] <= 1e-2, c
    assert orc.compare(lse.cpu().numpy(), rl)["max_abs"] <= 1e-3
