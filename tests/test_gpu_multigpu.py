"""Multi-GPU paths on real GPUs (skipped with fewer than 2 devices).

* Sequence-sharded split-KV decode: each rank holds a contiguous chunk of
  the KV cache, runs pu_decode_partial, the packed (m, l, o) partials move
  with one NCCL all-gather, and pu_decode_combine merges them; every rank
  must match the oracle's whole-cache decode.
* The same decode over NVLink peer memory (pu_decode_push / pu_decode_pull,
  no collective): bit-identical to the NCCL path over consecutive steps
  (both exchange slots), and a merge whose peers never publish runs out of
  its bounded wait, is reported (PU_ERR_DEVICE_TIMEOUT, detail 304), and
  leaves the context usable.
* Output projection fused with the TP all-reduce (pu_outproj_allreduce):
  every rank's result equals the fp32 sum of all ranks' products (bf16
  tolerance) and is bitwise identical across ranks, over consecutive calls.
* Head-partitioned training attention: each rank runs forward + backward
  on its heads only (no collective); the gathered outputs match the oracle.
Runs world_size 2 as spawned processes with NCCL_NVLS_ENABLE=0.
"""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "pallas-unbound_b200"), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

pytestmark = pytest.mark.gpu


def _worker(rank, world, store, out_dir):
    import torch.distributed as dist
    from helpers import randn
    from oracle import attention as orc
    from pallas_flash.kernels.decoding import pallas_flash_decoding
    from pallas_flash.ops.interface import flash_attention_backward, flash_attention_forward

    torch.cuda.set_device(rank)
    # the ranks meet through a store file (no TCP port to collide with one
    # that another process still holds)
    dist.init_process_group("nccl", init_method="file://" + store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    res = {}
    # --- sequence-sharded decode ---
    B, H, N, D = 2, 8, 8192, 128
    q = randn((B, H, 1, D), 71, dtype=torch.float16)
    k = randn((B, H, N, D), 72, dtype=torch.float16)
    v = randn((B, H, N, D), 73, dtype=torch.float16)
    lens = torch.tensor([N, 5000], dtype=torch.int32)
    n = N // world
    ks = k[:, :, rank * n:(rank + 1) * n].contiguous().cuda()
    vs = v[:, :, rank * n:(rank + 1) * n].contiguous().cuda()
    o, lse = pallas_flash_decoding(q.cuda(), ks, vs, kv_lens=lens.cuda(), group=dist.group.WORLD,
                                   return_lse=True)
    ro, rl = orc.decode_forward(q.float().numpy(), k.float().numpy(), v.float().numpy(), kv_lens=lens.numpy())
    res["dec_o"] = orc.compare(o.float().cpu().numpy(), ro)
    res["dec_lse"] = orc.compare(lse.cpu().numpy(), rl)
    # --- the same decode over peer memory, several steps ---
    from pallas_flash import _lib
    from pallas_flash.distributed import peer
    same = True
    for step in range(5):
        qs = randn((B, H, 1, D), 90 + step, dtype=torch.float16).cuda()
        o_n, l_n = pallas_flash_decoding(qs, ks, vs, kv_lens=lens.cuda(), group=dist.group.WORLD,
                                         return_lse=True)
        o_p, l_p = pallas_flash_decoding(qs, ks, vs, kv_lens=lens.cuda(), group=dist.group.WORLD,
                                         transport="peer", return_lse=True)
        same &= bool(torch.equal(o_n, o_p)) and bool(torch.equal(l_n, l_p))
    res["peer_equal"] = same
    res["peer_status"] = list(_lib.device_status())
    # --- the same decode through the library's own NCCL communicator ---
    from pallas_flash.distributed.collectives import close_lib_comms
    same_lib = True
    for step in range(3):
        qs = randn((B, H, 1, D), 120 + step, dtype=torch.float16).cuda()
        o_n, l_n = pallas_flash_decoding(qs, ks, vs, kv_lens=lens.cuda(), group=dist.group.WORLD,
                                         return_lse=True)
        o_l, l_l = pallas_flash_decoding(qs, ks, vs, kv_lens=lens.cuda(), group=dist.group.WORLD,
                                         transport="lib", return_lse=True)
        same_lib &= bool(torch.equal(o_n, o_l)) and bool(torch.equal(l_n, l_l))
    close_lib_comms()
    res["lib_equal"] = same_lib
    ex = peer.get_exchange(B, H, D, dist.group.WORLD)
    o_t = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device="cuda")
    # an epoch no rank will publish: the wait must run out (50 ms) and report
    _lib.check(_lib.lib().pu_decode_pull(ex._local, world, ex.epoch + 1000, o_t.data_ptr(), None,
                                         B, H, D, 50_000_000, torch.cuda.current_stream().cuda_stream),
               "pu_decode_pull")
    res["timeout_status"] = list(_lib.device_status())
    o_p, _ = pallas_flash_decoding(q.cuda(), ks, vs, kv_lens=lens.cuda(), group=dist.group.WORLD,
                                   transport="peer", return_lse=True)
    res["after_timeout"] = orc.compare(o_p.float().cpu().numpy(), ro)
    # --- output projection + TP all-reduce over peer memory ---
    from pallas_flash.distributed.outproj import out_proj_all_reduce
    T, Kl, Nm = 1024, 256, 1024
    worst = 0.0
    for step in range(3):
        os_ = [randn((T, Kl), 200 + 10 * step + g) for g in range(world)]
        ws_ = [(randn((Kl, Nm), 300 + 10 * step + g).float() / Kl ** 0.5).to(torch.bfloat16)
               for g in range(world)]
        y = out_proj_all_reduce(os_[rank].cuda(), ws_[rank].cuda(), dist.group.WORLD)
        ref = sum(os_[g].float() @ ws_[g].float() for g in range(world))
        yc = y.float().cpu()
        err = (yc - ref).abs().max().item() / ref.abs().max().item()
        rel = ((yc - ref).norm() / ref.norm()).item()
        worst = max(worst, err, rel)
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        res["outproj_same"] = all(torch.equal(ys[0], t) for t in ys)
    res["outproj_err"] = worst
    res["outproj_status"] = list(_lib.device_status())
    peer.close_all()
    # --- head-partitioned training attention ---
    B, H, N, D = 1, 4, 512, 128
    qg, kg, vg, dog = (randn((B, H, N, D), 80 + i) for i in range(4))
    hs = H // world
    sl = slice(rank * hs, (rank + 1) * hs)
    ql, kl, vl, dol = (t[:, sl].contiguous().cuda() for t in (qg, kg, vg, dog))
    ol, lsel = flash_attention_forward(ql, kl, vl, causal=True)
    dql, dkl, dvl = flash_attention_backward(ql, kl, vl, ol, lsel, dol, causal=True)
    f = lambda t: t.float().numpy()
    ro, rl = orc.mha_forward(f(qg)[:, sl], f(kg)[:, sl], f(vg)[:, sl], causal=True)
    rdq, rdk, rdv = orc.mha_backward(f(qg)[:, sl], f(kg)[:, sl], f(vg)[:, sl], ro, rl, f(dog)[:, sl], causal=True)
    res["tr_o"] = orc.compare(ol.float().cpu().numpy(), ro)
    for name, got, ref in (("dq", dql, rdq), ("dk", dkl, rdk), ("dv", dvl, rdv)):
        res["tr_" + name] = orc.compare(got.float().cpu().numpy(), ref)
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    import json
    Path(out_dir, f"rank{rank}.json").write_text(json.dumps(res))


def test_two_gpu_decode_and_partitioned_training(tmp_path, built_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import json
    import torch.multiprocessing as mp
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.start_processes(_worker, args=(2, str(tmp_path / "pg_store"), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    for rank in range(2):
        res = json.loads(Path(tmp_path, f"rank{rank}.json").read_text())
        assert res["dec_o"]["max_abs"] <= 2e-2 and res["dec_o"]["rel"] <= 1e-2, res
        assert res["dec_lse"]["max_abs"] <= 1e-3, res
        assert res["peer_equal"] and res["peer_status"] == [0, 0], res
        assert res["lib_equal"], res
        assert res["timeout_status"] == [5, 304], res
        assert res["after_timeout"]["max_abs"] <= 2e-2 and res["after_timeout"]["rel"] <= 1e-2, res
        assert res["outproj_same"] and res["outproj_err"] <= 1e-2 and res["outproj_status"] == [0, 0], res
        assert res["tr_o"]["max_abs"] <= 2e-2 and res["tr_o"]["rel"] <= 1e-2, res
        for g in ("dq", "dk", "dv"):
            assert res["tr_" + g]["rel"] <= 3e-2, res
