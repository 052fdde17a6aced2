"""Multi-rank host logic on CPU (torch.distributed, gloo, world_size 2).

Covers what the GPU runs do across ranks, without GPUs:
  * the ('dp','tp') head/batch partition (the reference's
    tests/test_distributed.py:52-86 expectations) and that per-rank attention
    on the partition reassembles the global result (no collective needed);
  * the sequence-sharded decode exchange: every rank computes its shard's
    packed (m, l, o) partial, all_gather_partials moves them, the stable
    merge reproduces the whole-cache decode;
  * failure detection on the host: a rank that leaves before the collective
    makes the survivor's all-gather fail with an error after the process
    group timeout instead of hanging.
"""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "pallas-unbound_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle import attention as orc  # noqa: E402
from pallas_flash.distributed import collectives, mesh  # noqa: E402


def rendezvous() -> str:
    """Store-file URL for one multi-process group (no TCP port to collide
    with one that another process still holds)."""
    import tempfile
    return "file://" + os.path.join(tempfile.mkdtemp(prefix="pu_pg_"), "store")


def _init(rank, world, url, timeout_s=30):
    dist.init_process_group("gloo", init_method=url, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def test_mesh_partition_matches_reference_expectations():
    # 1x4 mesh: heads over tp -> local (2, 4, 128, 64)  (test_distributed.py:69-84)
    m = mesh.create_mesh(4, dp_size=1, tp_size=4)
    x = torch.zeros(2, 16, 128, 64)
    for r in range(4):
        assert tuple(mesh.local_attention_shard(x, m, r).shape) == (2, 4, 128, 64)
    # 4x1 mesh: batch over dp (test_distributed.py:131-153)
    m = mesh.create_mesh(4, dp_size=4, tp_size=1)
    x = torch.zeros(8, 16, 128, 64)
    assert tuple(mesh.local_attention_shard(x, m, 3).shape) == (2, 16, 128, 64)
    # too few devices: fall back to 1 x world (mesh.py:44-50)
    assert mesh.create_mesh(2, dp_size=2, tp_size=4) == mesh.Mesh(1, 2)


def test_partitioned_attention_reassembles_global_result():
    rng = np.random.Generator(np.random.PCG64(7))
    q, k, v = (orc.bf16_round(rng.standard_normal((2, 4, 64, 32), dtype=np.float32)) for _ in range(3))
    go, _ = orc.mha_forward(q, k, v, causal=True)
    m = mesh.create_mesh(4, dp_size=2, tp_size=2)
    out = np.zeros_like(go)
    for r in range(4):
        d, t = m.coords(r)
        lq, lk, lv = (mesh.local_attention_shard(torch.from_numpy(a), m, r).numpy() for a in (q, k, v))
        lo, _ = orc.mha_forward(lq, lk, lv, causal=True)
        out[d:d + 1, 2 * t:2 * t + 2] = lo
    np.testing.assert_allclose(out, go, atol=1e-12)


def _decode_exchange(rank, world, port, result_path):
    _init(rank, world, port)
    rng = np.random.Generator(np.random.PCG64(11))
    B, H, N, D = 2, 3, 512, 64
    q = rng.standard_normal((B, H, 1, D)).astype(np.float16)
    k = rng.standard_normal((B, H, N, D)).astype(np.float16)
    v = rng.standard_normal((B, H, N, D)).astype(np.float16)
    lens = np.array([N, 100])
    ks = collectives.sequence_shard(torch.from_numpy(k), rank, world).numpy()
    vs = collectives.sequence_shard(torch.from_numpy(v), rank, world).numpy()
    part = orc.decode_partial(q, ks, vs, kv_offset=rank * (N // world), kv_lens=lens)
    gathered = collectives.all_gather_partials(torch.from_numpy(part), world)
    o, lse = orc.lse_combine(gathered.numpy())
    ro, rl = orc.decode_forward(q, k, v, kv_lens=lens)
    ok = np.allclose(o.reshape(ro.shape), ro, atol=1e-10) and np.allclose(lse.reshape(rl.shape), rl, atol=1e-10)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        Path(result_path).write_text("ok" if ok else "mismatch")


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_sharded_decode_exchange(tmp_path, world):
    res = tmp_path / "res.txt"
    mp.start_processes(_decode_exchange, args=(world, rendezvous(), str(res)), nprocs=world,
                       start_method="spawn", join=True)
    assert res.read_text() == "ok"


def _leaver(rank, world, port, result_path):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # leaves between steps: no collective of this step is ever entered
        dist.destroy_process_group()
        return
    part = torch.zeros(3, 10)
    t0 = datetime.datetime.now()
    try:
        collectives.all_gather_partials(part, world)
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - any collective error is the detection
        outcome = f"error after {(datetime.datetime.now() - t0).total_seconds():.1f}s: {type(e).__name__}"
    Path(result_path).write_text(outcome)


def test_lost_rank_is_detected_not_hung(tmp_path):
    res = tmp_path / "res.txt"
    ctx = mp.start_processes(_leaver, args=(2, rendezvous(), str(res)), nprocs=2,
                             start_method="spawn", join=False)
    deadline = 90
    t0 = datetime.datetime.now()
    while not ctx.join(timeout=1):
        assert (datetime.datetime.now() - t0).total_seconds() < deadline, "survivor hung"
    assert res.read_text().startswith("error after"), res.read_text()


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_length_balanced_split_covers_every_token_once(world):
    """Every held token of every sequence goes to exactly one rank, in
    contiguous per-rank slices; per-rank totals differ by a few blocks at
    most (the blocks left over by the integer split rotate over ranks)."""
    rng = np.random.Generator(np.random.PCG64(4))
    lens = (np.ceil(rng.uniform(4096, 131072, size=8) / 128) * 128).astype(np.int64)
    lens[3] = 0
    lens[5] = 77            # a tail shorter than one granule
    starts, counts = collectives.length_balanced_split(lens, world, granule=128)
    assert starts.shape == counts.shape == (world, 8)
    for b in range(8):
        seen = np.zeros(lens[b], dtype=np.int64)
        for r in range(world):
            seen[starts[r, b]:starts[r, b] + counts[r, b]] += 1
            if r + 1 < world:
                assert starts[r + 1, b] == starts[r, b] + counts[r, b]
        assert (seen == 1).all()
    tot = counts.sum(axis=1)
    assert tot.max() - tot.min() <= 3 * 128          # a few blocks, whatever the raggedness
    assert tot.max() <= 1.01 * tot.mean()


def test_length_balanced_shards_merge_to_whole_cache_decode():
    """Per-rank partials over length-balanced shards (local lengths, no
    offset) merge to the decode over the whole ragged cache."""
    rng = np.random.Generator(np.random.PCG64(12))
    B, H, N, D, G = 3, 2, 700, 64, 4
    q = rng.standard_normal((B, H, 1, D)).astype(np.float32)
    k = rng.standard_normal((B, H, N, D)).astype(np.float32)
    v = rng.standard_normal((B, H, N, D)).astype(np.float32)
    lens = np.array([700, 129, 1])
    ref_o, ref_lse = orc.decode_forward(q, k, v, kv_lens=lens)
    parts = []
    for r in range(G):
        kl, vl, ll = collectives.shard_by_length(torch.from_numpy(k), torch.from_numpy(v), lens, r, G,
                                                 granule=128)
        parts.append(orc.decode_partial(q, kl.numpy(), vl.numpy(), kv_offset=0, kv_lens=ll.numpy()))
    o, lse = orc.lse_combine(np.stack(parts))
    assert np.abs(o.reshape(ref_o.shape) - ref_o).max() < 1e-5
    assert np.abs(lse.reshape(ref_lse.shape) - ref_lse).max() < 1e-5
