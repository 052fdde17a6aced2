#!/usr/bin/env python
"""Benchmark of the B200 attention hot path (one JSON line on stdout).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl pu|reference]

Headline workload (one "step", per GPU): causal flash-attention training
forward + backward, B=4, H=16, N=4096, D=128, bf16, Q/K/V/dO ~ N(0,1)
(the reference's training-attention configuration).  Under torchrun each
rank owns its own 16 heads (heads are independent: no collective), so the
per-GPU work is fixed and the job scales weakly; `value` is the aggregate
TFLOP/s of all ranks, FLOPs counted as 4*B*H*N^2*D/2 forward (causal) and
2.5x that backward (the reference's convention, benchmarks/scaling.py:44-54).

The same line carries the split-KV decode measurement (B=1, H=32, a
32768-token fp16 KV cache sharded by sequence over the N GPUs, NCCL
all-gather of the (m, l, o) partials, fused LSE combine) as `decode`.

Before any timed leg every rank checks small seeded cases of each path it
runs against the oracle (head-partitioned causal fwd+bwd, the
sequence-sharded decode over each transport, the length-balanced ragged
decode, the fused out-projection) and the line carries the worst errors over
the ranks as `parity`; a miss makes the run exit non-zero after printing.

`--impl reference` times the reference algorithm on the host CPU instead
(the numpy restatement in oracle/, since the JAX reference cannot run
here) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "pallas-unbound_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "attn fwd+bwd TFLOP/s (% BF16 peak); split-KV decode µs/step, HBM GB/s @1-8 GPU"
B, H, N, D = 4, 16, 4096, 128
DEC_B, DEC_H, DEC_N, DEC_D = 1, 32, 32768, 128
FWD_FLOPS = 4 * B * H * N * N * D * 0.5          # causal
STEP_FLOPS = FWD_FLOPS * 3.5                      # fwd + 2.5x bwd
L2_BYTES = 126 * 1024 * 1024
# DRAM bytes (read + write) per launch of this workload, from one ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum) of
# `python bench.py --profile-leg attn --steps 2 --warmup 3` on one B200, the
# command and date in TRAFFIC_CAPTURE; re-captured whenever a kernel changes.
NCU_TRAFFIC_BYTES = {
    "attn_fwd": 523_139_584 + 49_843_712,
    # prep (135.3 + 84.0 MB) + fused backward (404.8 + 218.1 MB) + dQ conversion (134.2 + 32.5 MB)
    "attn_bwd": (135_290_368 + 83_952_384) + (404_835_840 + 218_139_136) + (134_240_000 + 32_545_792),
    "split_kv": 536_904_192 + 3_470_848,
}
TRAFFIC_CAPTURE = ("ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none "
                   "-k regex:'attn_fwd|prep_kernel|attn_bwd_fused|dq_convert' -s 12 -c 4 "
                   "python bench.py --profile-leg attn --steps 2 --warmup 3 (2026-12-02)")


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML, read-only)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples: list[tuple[float, int, int]] = []
        self.period = period_s
        self._stop = threading.Event()
        self._window = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: no clock record
            self._nv = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM)
                rs = self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self._nv is not None:
            self._t.start()
        return self

    def mark(self, t0, t1):
        self._window = (t0, t1)

    def stop(self) -> dict:
        if self._nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        self._stop.set()
        self._t.join(timeout=2)
        win = [s for s in self.samples if self._window and self._window[0] <= s[0] <= self._window[1]]
        used = win if win else self.samples
        mhz = [s[1] for s in used]
        bits = 0
        for s in used:
            bits |= s[2]
        reasons = sorted({name for bit, name in self.REASONS.items() if bits & bit and name != "gpu_idle"})
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(used), "in_window": bool(win)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_init():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


_ALIGN = {}


def device_align(world: int):
    """Align the ranks on the device before a timed multi-GPU step: a 1-element
    NCCL all-reduce on the current stream completes on every GPU at nearly the
    same moment, so the start events that follow it are not skewed by how long
    each GPU's preceding (untimed) work took."""
    if world > 1:
        import torch
        import torch.distributed as dist
        t = _ALIGN.get("t")
        if t is None:
            t = _ALIGN["t"] = torch.zeros(1, device="cuda")
        dist.all_reduce(t)


# ---------------------------------------------------------------------------
# CPU baselines (rank 0, N=1, bounded samples of the same workloads)
# ---------------------------------------------------------------------------
def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return max(n)
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_attention_sample(heads: int = 2):
    """Oracle fwd+bwd (numpy fp32) on `heads` heads of the B=4 H=16 N=4096 D=128 workload."""
    import numpy as np
    from oracle import attention as orc
    rng = np.random.Generator(np.random.PCG64(1))
    q = rng.standard_normal((1, heads, N, D), dtype=np.float32)
    k = rng.standard_normal((1, heads, N, D), dtype=np.float32)
    v = rng.standard_normal((1, heads, N, D), dtype=np.float32)
    do = rng.standard_normal((1, heads, N, D), dtype=np.float32)
    t0 = time.perf_counter()
    o, lse = orc.mha_forward(q, k, v, causal=True, dtype=np.float32, row_chunk=N)
    orc.mha_backward(q, k, v, o, lse, do, causal=True, dtype=np.float32, row_chunk=N)
    dt = time.perf_counter() - t0
    flops = STEP_FLOPS * heads / (B * H)
    return flops / dt / 1e12, dt, f"{heads} of {B * H} (b,h) heads of the causal B4 H16 N4096 D128 fwd+bwd, numpy fp32"


def cpu_decode_sample(heads: int = 8):
    import numpy as np
    from oracle import attention as orc
    rng = np.random.Generator(np.random.PCG64(3))
    q = rng.standard_normal((1, heads, 1, DEC_D)).astype(np.float16)
    k = rng.standard_normal((1, heads, DEC_N, DEC_D)).astype(np.float16)
    v = rng.standard_normal((1, heads, DEC_N, DEC_D)).astype(np.float16)
    reps = 3
    t0 = time.perf_counter()
    for _ in range(reps):
        orc.decode_forward(q, k, v, dtype=np.float32)
    dt = (time.perf_counter() - t0) / reps
    us_full = dt * 1e6 * DEC_H / heads
    return us_full, f"{heads} of {DEC_H} heads of the 32768-token fp16 decode, numpy fp32, scaled to 32 heads"


# ---------------------------------------------------------------------------
# Parity of every measured path on small seeded cases (the oracle is the
# checker; nothing here is timed)
# ---------------------------------------------------------------------------
PARITY_TOL = {"o_max_abs": 2e-2, "o_rel": 1e-2, "lse_abs": 1e-3, "grad_rel": 3e-2}


def single_rank_group():
    """A one-rank gloo group (the peer-memory entry points take a group even
    when there is nothing to exchange)."""
    import torch.distributed as dist
    if not dist.is_initialized():
        import tempfile
        store = os.path.join(tempfile.mkdtemp(prefix="pu_pg_"), "store")
        dist.init_process_group("gloo", init_method="file://" + store, rank=0, world_size=1)
    return dist.group.WORLD


def run_parity(rank: int, world: int) -> dict:
    """Small seeded cases of each path against the oracle on every rank;
    returns {case: {max_abs, rel, ok}} with the worst value over the ranks.

    * attn_fwd_bwd: causal B=1, 2 heads per rank (heads partitioned as in the
      timed leg), N=384, D=128; O and LSE, then dQ/dK/dV.
    * decode_<transport>: B=1 H=8, 1024 cache tokens per rank (sequence
      shards of one 1024*world-token fp16 cache) over each transport.
    * decode_ragged_by_length: B=3 H=4 with lengths 5000/1300/129 split over
      the ranks by held tokens.
    * outproj_<transport>: y = sum over ranks of o_r [256, 256] @ w_r [256, 256].
    """
    import numpy as np
    import torch
    from oracle import attention as orc
    from pallas_flash.distributed import collectives
    from pallas_flash.distributed.outproj import out_proj_all_reduce
    from pallas_flash.kernels import decoding as dec
    from pallas_flash.ops import interface as pf

    f = lambda t: t.detach().float().cpu().numpy()
    out = {}

    def rec(name, actual, expected, rel_tol, abs_tol=None):
        r = orc.compare(actual, expected)
        out[name] = [r["max_abs"], r["rel"], rel_tol, abs_tol]

    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    # head-partitioned causal forward + backward
    rng = np.random.Generator(np.random.PCG64(101))
    Hg, Np, Dp = 2 * world, 384, 128
    full = [rng.standard_normal((1, Hg, Np, Dp), dtype=np.float32) for _ in range(4)]
    loc = [torch.from_numpy(x[:, 2 * rank:2 * rank + 2].copy()).to(torch.bfloat16) for x in full]
    q, k, v, do = (t.cuda() for t in loc)
    o, lse = pf.flash_attention_forward(q, k, v, causal=True)
    dq, dk, dv = pf.flash_attention_backward(q, k, v, o, lse, do, causal=True)
    qn, kn, vn, don = (f(t) for t in loc)
    ro, rl = orc.mha_forward(qn, kn, vn, causal=True)
    rdq, rdk, rdv = orc.mha_backward(qn, kn, vn, ro, rl, don, causal=True)
    rec("attn_fwd_o", f(o), ro, PARITY_TOL["o_rel"], PARITY_TOL["o_max_abs"])
    rec("attn_fwd_lse", f(lse), rl, float("inf"), PARITY_TOL["lse_abs"])
    for name, got, ref in (("attn_bwd_dq", dq, rdq), ("attn_bwd_dk", dk, rdk), ("attn_bwd_dv", dv, rdv)):
        rec(name, f(got), ref, PARITY_TOL["grad_rel"])
    # sequence-sharded decode over each transport
    rng = np.random.Generator(np.random.PCG64(102))
    Bd, Hd, nl, Dd = 1, 8, 1024, 128
    qd = torch.from_numpy(rng.standard_normal((Bd, Hd, 1, Dd), dtype=np.float32)).half()
    kd = torch.from_numpy(rng.standard_normal((Bd, Hd, nl * world, Dd), dtype=np.float32)).half()
    vd = torch.from_numpy(rng.standard_normal((Bd, Hd, nl * world, Dd), dtype=np.float32)).half()
    ro, rl = orc.decode_forward(f(qd), f(kd), f(vd))
    kl = kd[:, :, rank * nl:(rank + 1) * nl].contiguous().cuda()
    vl = vd[:, :, rank * nl:(rank + 1) * nl].contiguous().cuda()
    transports = ("peer", "nccl", "lib") if world > 1 else ("single",)
    for t in transports:
        kw = {"group": group, "transport": t} if world > 1 else {}
        o, lse = dec.pallas_flash_decoding(qd.cuda(), kl, vl, return_lse=True, **kw)
        rec(f"decode_{t}_o", f(o), ro, PARITY_TOL["o_rel"], PARITY_TOL["o_max_abs"])
        rec(f"decode_{t}_lse", f(lse), rl, float("inf"), PARITY_TOL["lse_abs"])
    # ragged batch sharded by held tokens
    rng = np.random.Generator(np.random.PCG64(103))
    lens = np.array([5000, 1300, 129])
    Br, Hr, Nr = 3, 4, 5120
    qr = torch.from_numpy(rng.standard_normal((Br, Hr, 1, Dd), dtype=np.float32)).half()
    kr = torch.from_numpy(rng.standard_normal((Br, Hr, Nr, Dd), dtype=np.float32)).half()
    vr = torch.from_numpy(rng.standard_normal((Br, Hr, Nr, Dd), dtype=np.float32)).half()
    ro, rl = orc.decode_forward(f(qr), f(kr), f(vr), kv_lens=lens)
    if world > 1:
        kl, vl, ll = collectives.shard_by_length(kr, vr, lens, rank, world)
        o = dec.pallas_flash_decoding(qr.cuda(), kl.cuda(), vl.cuda(), kv_lens=ll.cuda(), group=group,
                                      transport="peer", sharding="by_length")
    else:
        o = dec.pallas_flash_decoding(qr.cuda(), kr.cuda(), vr.cuda(),
                                      kv_lens=torch.from_numpy(lens).cuda())
    rec("decode_ragged_by_length_o", f(o), ro, PARITY_TOL["o_rel"], PARITY_TOL["o_max_abs"])
    # fused out-projection + all-reduce
    To, Ko, No = 256, 256, 256
    ows = []
    for r in range(world):
        g = np.random.Generator(np.random.PCG64(200 + r))
        ows.append((torch.from_numpy(g.standard_normal((To, Ko), dtype=np.float32)).to(torch.bfloat16),
                    torch.from_numpy(g.standard_normal((Ko, No), dtype=np.float32) / Ko ** 0.5)
                    .to(torch.bfloat16)))
    yref = sum(f(a).astype(np.float64) @ f(b).astype(np.float64) for a, b in ows)
    grp = group if world > 1 else single_rank_group()
    for t in (("peer", "nccl") if world > 1 else ("peer",)):
        y = out_proj_all_reduce(ows[rank][0].cuda(), ows[rank][1].cuda(), grp, transport=t)
        rec(f"outproj_{t}", f(y), yref, PARITY_TOL["o_rel"], 2e-2 * float(np.abs(yref).max()))
    torch.cuda.synchronize()
    from pallas_flash import _lib
    code, detail = _lib.device_status()
    if code != 0:
        raise RuntimeError(f"device status {code} at site {detail} during the parity checks")
    # worst over the ranks
    names = sorted(out)
    vals = torch.tensor([[out[n][0], out[n][1]] for n in names], dtype=torch.float64, device="cuda")
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    res = {}
    for i, n in enumerate(names):
        mx, rel = float(vals[i, 0]), float(vals[i, 1])
        rel_tol, abs_tol = out[n][2], out[n][3]
        ok = rel <= rel_tol and (abs_tol is None or mx <= abs_tol)
        res[n] = {"max_abs": float(f"{mx:.3g}"), "rel": float(f"{rel:.3g}"), "ok": bool(ok)}
    return res


# ---------------------------------------------------------------------------
# GPU measurements
# ---------------------------------------------------------------------------
def bench_attention(steps: int, warmup: int, rank: int, world: int, clocks: ClockSampler, batch: int = B):
    import torch
    from pallas_flash.ops import interface as pf

    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + rank)
    shape = (batch, H, N, D)
    q, k, v, do = (torch.randn(shape, device="cuda", dtype=torch.float32, generator=g).to(torch.bfloat16)
                   for _ in range(4))
    o = torch.empty_like(q)
    lse = torch.empty((batch, H, N), device="cuda", dtype=torch.float32)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws = torch.empty(pf.bwd_workspace_bytes(batch, H, N, D), device="cuda", dtype=torch.uint8)
    stream = torch.cuda.current_stream()

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        pf.flash_attention_forward(q, k, v, causal=True, out=o, lse=lse)
        if ev is not None:
            ev[1].record(stream)
        pf.flash_attention_backward(q, k, v, o, lse, do, causal=True, workspace=ws, dq=dq, dk=dk, dv=dv)
        if ev is not None:
            ev[2].record(stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    start.record(stream)
    for i in range(steps):
        step(evs[i])
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier(world)
    clocks.mark(t0, t1)
    total_ms = start.elapsed_time(end)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
    from pallas_flash import _lib
    code, detail = _lib.device_status()
    if code != 0:
        raise RuntimeError(f"device status {code} at site {detail}")
    return total_ms, fwd_ms, bwd_ms


C1_B, C1_H, C1_N = 1, 4, 1024
C1_FLOPS = 4 * C1_B * C1_H * C1_N * C1_N * D * 0.5        # causal


def bench_c1(steps: int, warmup: int) -> float:
    """Causal forward B=1 H=4 N=1024 D=128 (the reference's CPU baseline_mha
    configuration) on one GPU: median microseconds per call, L2 flushed
    before every call (the inputs, 3 MB, would otherwise stay in L2)."""
    import torch
    from pallas_flash.ops import interface as pf

    g = torch.Generator(device="cuda")
    g.manual_seed(7000)
    shape = (C1_B, C1_H, C1_N, D)
    q, k, v = (torch.randn(shape, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    lse = torch.empty((C1_B, C1_H, C1_N), device="cuda", dtype=torch.float32)

    def step():
        pf.flash_attention_forward(q, k, v, causal=True, out=o, lse=lse)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    lat = _timed(step, steps, L2Flush(), torch.cuda.current_stream())
    ring = [(q, k, v)] + [(q.clone(), k.clone(), v.clone()) for _ in range(_copies(3 * q.numel() * 2) - 1)]
    us = _steady(lambda t: pf.flash_attention_forward(t[0], t[1], t[2], causal=True, out=o, lse=lse),
                 ring, max(steps, len(ring)), warmup, torch.cuda.current_stream())
    return us, lat, len(ring)


def cpu_c1_sample():
    """The oracle's causal baseline_mha restatement (numpy fp32) on the c1
    shape: best of 3 runs, seconds."""
    import numpy as np
    from oracle import attention as orc
    rng = np.random.Generator(np.random.PCG64(7))
    q, k, v = (rng.standard_normal((C1_B, C1_H, C1_N, D), dtype=np.float32) for _ in range(3))
    best = float("inf")
    for _ in range(3):
        t0 = time.perf_counter()
        orc.mha_forward(q, k, v, causal=True, dtype=np.float32, row_chunk=C1_N)
        best = min(best, time.perf_counter() - t0)
    return best


LONG_B, LONG_H, LONG_N = 1, 32, 16384
LONG_FWD_FLOPS = 4 * LONG_B * LONG_H * LONG_N * LONG_N * D      # non-causal


def bench_attention_long(steps: int, warmup: int):
    """Non-causal long-sequence fwd+bwd on one GPU: B=1, H=32, N=16384,
    D=128, Q/K/V ~ N(0, 0.5), dO ~ N(0, 1) (bf16).  Returns (fwd_ms, bwd_ms)
    per step (medians)."""
    import torch
    from pallas_flash.ops import interface as pf

    g = torch.Generator(device="cuda")
    g.manual_seed(3000)
    shape = (LONG_B, LONG_H, LONG_N, D)
    q, k, v = ((torch.randn(shape, device="cuda", generator=g) * 0.5).to(torch.bfloat16) for _ in range(3))
    do = torch.randn(shape, device="cuda", generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty((LONG_B, LONG_H, LONG_N), device="cuda", dtype=torch.float32)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws = torch.empty(pf.bwd_workspace_bytes(LONG_B, LONG_H, LONG_N, D), device="cuda", dtype=torch.uint8)
    stream = torch.cuda.current_stream()
    fwd, bwd = [], []
    for i in range(warmup + steps):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        e[0].record(stream)
        pf.flash_attention_forward(q, k, v, causal=False, out=o, lse=lse)
        e[1].record(stream)
        pf.flash_attention_backward(q, k, v, o, lse, do, causal=False, workspace=ws, dq=dq, dk=dk, dv=dv)
        e[2].record(stream)
        torch.cuda.synchronize()
        if i >= warmup:
            fwd.append(e[0].elapsed_time(e[1]))
            bwd.append(e[1].elapsed_time(e[2]))
    from pallas_flash import _lib
    code, detail = _lib.device_status()
    if code != 0:
        raise RuntimeError(f"device status {code} at site {detail}")
    return statistics.median(fwd), statistics.median(bwd)


def bench_attention_e2e(steps: int, warmup: int, rank: int, world: int):
    """Through the public API with host (pinned) tensors: H2D of q, k, v, dO and
    D2H of o, dq, dk, dv inside every timed step (torch.autograd drives the
    backward through pallas_flash_attention)."""
    import torch
    from pallas_flash.ops.interface import pallas_flash_attention

    g = torch.Generator()
    g.manual_seed(2000 + rank)
    shape = (B, H, N, D)
    host = [torch.randn(shape, generator=g).to(torch.bfloat16).pin_memory() for _ in range(4)]
    qh, kh, vh, doh = host
    for t in (qh, kh, vh):
        t.requires_grad_(True)

    def step():
        for t in (qh, kh, vh):
            t.grad = None
        o = pallas_flash_attention(qh, kh, vh, causal=True)    # H2D q,k,v ; D2H o
        o.backward(doh)                                         # H2D dO ; D2H dq,dk,dv
        return o

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) / steps
    dt = allreduce_max(dt, world)
    nbytes = qh.numel() * 2
    return dt, 4 * nbytes, 4 * nbytes


def bench_decode(steps: int, warmup: int, rank: int, world: int, transport: str = "peer"):
    """Decode step time (median over single steps after an L2 flush, max over
    ranks), kernel-only time of the local split-KV pass, the K/V bytes one rank
    reads, the steady-state time per step of back-to-back steps over rotating
    cache copies (max over ranks) and the number of copies.  With more than
    one rank the partials travel by `transport` ("peer": NVLink peer stores +
    flags; "nccl": all-gather)."""
    import torch
    from pallas_flash.kernels import decoding as dec

    n_local = DEC_N // world
    g = torch.Generator(device="cuda")
    g.manual_seed(3000 + rank)
    q = torch.randn((DEC_B, DEC_H, 1, DEC_D), device="cuda", generator=g).to(torch.float16)
    k = torch.randn((DEC_B, DEC_H, n_local, DEC_D), device="cuda", generator=g).to(torch.float16)
    v = torch.randn((DEC_B, DEC_H, n_local, DEC_D), device="cuda", generator=g).to(torch.float16)
    flusher = L2Flush()
    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    stream = torch.cuda.current_stream()

    def step():
        return dec.pallas_flash_decoding(q, k, v, group=group, transport=transport)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    times = []
    for _ in range(steps):
        barrier(world)                              # ranks start each step together
        flusher()                                   # evict the cache shard from L2
        device_align(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    # steady state: `steps` steps back to back under one pair of events, each
    # step on the next of R cache copies, R * shard > 2 x L2, so no step finds
    # its shard in L2 (no flush, no per-step launch gap), the host ahead of
    # the device
    copies = max(1, -(-2 * L2_BYTES // (2 * k.numel() * k.element_size())))
    ring = [(k, v)] + [(k.clone(), v.clone()) for _ in range(copies - 1)]
    for i in range(warmup):
        dec.pallas_flash_decoding(q, *ring[i % copies], group=group, transport=transport)
    torch.cuda.synchronize()
    barrier(world)
    gpu_lead(steps)
    device_align(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        dec.pallas_flash_decoding(q, *ring[i % copies], group=group, transport=transport)
    e1.record(stream)
    torch.cuda.synchronize()
    steady = e0.elapsed_time(e1) * 1e3 / steps
    # kernel-only time of the local split-KV pass (pu_decode_partial / pu_decode),
    # the same way: back to back over the rotating copies
    part = torch.empty((DEC_B * DEC_H, DEC_D + 2), device="cuda", dtype=torch.float32)

    def local(i):
        kk, vv = ring[i % copies]
        if world == 1:
            dec.pallas_flash_decoding(q, kk, vv)
        else:
            dec.decode_partial(q, kk, vv, kv_offset=rank * n_local, out=part)
    for i in range(warmup):
        local(i)
    torch.cuda.synchronize()
    gpu_lead(steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        local(i)
    e1.record(stream)
    torch.cuda.synchronize()
    kern_steady = e0.elapsed_time(e1) * 1e3 / steps
    del ring
    barrier(world)
    us = allreduce_max(statistics.median(times) * 1e3, world)
    kus = allreduce_max(kern_steady, world)
    steady = allreduce_max(steady, world)
    return us, kus, 2 * DEC_B * DEC_H * n_local * DEC_D * 2, steady, copies


RAG_B, RAG_H, RAG_NCAP, RAG_D, RAG_PAGE = 8, 16, 131072, 128, 64


def ragged_lens():
    """Per-sequence lengths U[4096, 131072] rounded up to 128 (seeded)."""
    import numpy as np
    rng = np.random.Generator(np.random.PCG64(4))
    return (np.ceil(rng.uniform(4096, RAG_NCAP, size=RAG_B) / 128) * 128).astype(np.int32)


class L2Flush:
    """Evicts the L2 between timed decode steps: writes a 1 GiB buffer, then
    reads another 1 GiB buffer.  The read must be this large: after a 256 MB
    read, dirty lines of the write were still in L2 and the timed step paid
    their write-backs (+7 us on the 32k-token decode).  The ~0.3 ms of flush
    work also lets the host enqueue the step before the GPU reaches the start
    event, so the events time the device work only."""

    def __init__(self):
        import torch
        self.w = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
        self.r = torch.ones((1 << 30) // 4, dtype=torch.float32, device="cuda")
        self.acc = torch.zeros((), dtype=torch.float32, device="cuda")

    def __call__(self):
        import torch
        self.w.zero_()
        torch.sum(self.r, dim=0, out=self.acc)


def _timed(fn, steps, flush, stream, world: int = 1):
    import torch
    times = []
    for _ in range(steps):
        flush()
        device_align(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times) * 1e3


_LEAD = {}


def gpu_lead(steps: int):
    """Queues about 0.3 ms of device work (L2 flushes) per 6 steps ahead of a
    back-to-back timed loop, so the host has enqueued the steps before the
    device reaches them: the events then time device work only, for steps
    whose host-side call (~30 us) is as long as their device time."""
    f = _LEAD.get("flush")
    if f is None:
        f = _LEAD["flush"] = L2Flush()
    for _ in range(max(1, -(-steps // 6))):
        f()


def _steady(fn, ring, steps: int, warmup: int, stream, world: int = 1) -> float:
    """Microseconds per call of `steps` calls back to back under one pair of
    CUDA events, call i on ring[i % len(ring)] (the caller sizes the ring so
    its inputs exceed twice the L2: no call finds its inputs there), with
    the host ahead of the device (gpu_lead)."""
    import torch
    for i in range(warmup):
        fn(ring[i % len(ring)])
    torch.cuda.synchronize()
    barrier(world)
    gpu_lead(steps)
    device_align(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        fn(ring[i % len(ring)])
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / steps


def _copies(nbytes: int) -> int:
    """Copies of an input of `nbytes` whose total exceeds twice the L2."""
    return max(1, -(-2 * L2_BYTES // max(1, nbytes)))


def bench_ragged_decode(steps: int, warmup: int, rank: int, world: int):
    """Batched ragged decode (B=8, H=16, D=128, fp16, lengths U[4096, 131072]).
    One GPU: the dense padded cache, and the same tokens in a paged cache of
    64-token pages in shuffled order.  Several GPUs: every rank holds an equal
    slice of every sequence's held tokens (length-balanced sharding), and,
    for comparison, contiguous chunks of the padded capacity.
    Returns (dense us, paged us or None, contiguous us or None, algorithmic
    bytes of all ranks)."""
    import numpy as np
    import torch
    from pallas_flash.distributed import collectives
    from pallas_flash.kernels import decoding as dec
    from pallas_flash.kernels import paged

    lens = ragged_lens()
    g = torch.Generator(device="cuda")
    g.manual_seed(4000 + rank)
    q = torch.randn((RAG_B, RAG_H, 1, RAG_D), device="cuda", generator=g).to(torch.float16)
    flush = L2Flush()
    stream = torch.cuda.current_stream()
    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    nbytes = int(lens.astype(np.int64).sum()) * RAG_H * RAG_D * 2 * 2
    paged_us = contiguous_us = None
    if world == 1:
        k = torch.randn((RAG_B, RAG_H, RAG_NCAP, RAG_D), device="cuda", generator=g).to(torch.float16)
        v = torch.randn((RAG_B, RAG_H, RAG_NCAP, RAG_D), device="cuda", generator=g).to(torch.float16)
        lens_t = torch.from_numpy(lens).cuda()
        dense = lambda: dec.pallas_flash_decoding(q, k, v, kv_lens=lens_t)
    else:
        starts, counts = collectives.length_balanced_split(lens, world)
        cap = int(-(-int(counts.max()) // 128) * 128)
        k = torch.randn((RAG_B, RAG_H, cap, RAG_D), device="cuda", generator=g).to(torch.float16)
        v = torch.randn((RAG_B, RAG_H, cap, RAG_D), device="cuda", generator=g).to(torch.float16)
        lens_t = torch.from_numpy(counts[rank].astype(np.int32)).cuda()
        dense = lambda: dec.pallas_flash_decoding(q, k, v, kv_lens=lens_t, group=group, transport="peer",
                                                  sharding="by_length")
    for _ in range(warmup):
        dense()
    torch.cuda.synchronize()
    barrier(world)
    dense_us = allreduce_max(_timed(dense, steps, flush, stream, world), world)
    if world == 1:
        cache = paged.PagedKVCache.from_dense(k, v, lens, page_size=RAG_PAGE, shuffle_seed=1)
        del k, v

        def run_paged():
            return cache.decode(q)

        for _ in range(warmup):
            run_paged()
        torch.cuda.synchronize()
        paged_us = _timed(run_paged, steps, flush, stream)
    else:
        del k, v
        n_local = RAG_NCAP // world
        kc = torch.randn((RAG_B, RAG_H, n_local, RAG_D), device="cuda", generator=g).to(torch.float16)
        vc = torch.randn((RAG_B, RAG_H, n_local, RAG_D), device="cuda", generator=g).to(torch.float16)
        glens = torch.from_numpy(lens).cuda()
        contig = lambda: dec.pallas_flash_decoding(q, kc, vc, kv_lens=glens, group=group, transport="peer")
        for _ in range(warmup):
            contig()
        torch.cuda.synchronize()
        barrier(world)
        contiguous_us = allreduce_max(_timed(contig, steps, flush, stream, world), world)
        del kc, vc
    return dense_us, paged_us, contiguous_us, nbytes


OP_T, OP_K, OP_N = 4 * 4096, 16 * 128, 2048


def bench_outproj(steps: int, warmup: int, rank: int, world: int):
    """Attention output projection + TP all-reduce: every rank multiplies its
    16 heads' output [16384, 2048] by its rows of W_O [2048, 2048]; the
    partial products are summed over the ranks (weak scaling: K per rank is
    fixed).  Returns {transport: (us, latency_us, copies)} (max over ranks):
    us per call of `steps` calls back to back under one pair of events, call
    i reading copy i mod R of the activation (R copies exceed twice the L2);
    latency_us the median of single calls, each started on an idle GPU (so
    it includes the host-side work before the launch)."""
    import torch
    from pallas_flash.distributed.outproj import out_proj_all_reduce

    g = torch.Generator(device="cuda")
    g.manual_seed(6000 + rank)
    o = torch.randn((OP_T, OP_K), device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn((OP_K, OP_N), device="cuda", generator=g) / OP_K ** 0.5).to(torch.bfloat16)
    y = torch.empty((OP_T, OP_N), device="cuda", dtype=torch.bfloat16)
    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    else:
        group = single_rank_group()
    stream = torch.cuda.current_stream()
    ring = [o] + [o.clone() for _ in range(_copies(o.numel() * o.element_size()) - 1)]
    out = {}
    for transport in ("peer", "nccl"):
        if world == 1 and transport == "nccl":
            fn = lambda a: torch.matmul(a, w, out=y)
        else:
            fn = lambda a: out_proj_all_reduce(a, w, group, transport=transport, out=y)
        for _ in range(warmup):
            fn(o)
        torch.cuda.synchronize()
        barrier(world)
        times = []
        for _ in range(steps):
            barrier(world)
            device_align(world)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn(o)
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        lat = allreduce_max(statistics.median(times) * 1e3, world)
        us = allreduce_max(_steady(fn, ring, max(steps, len(ring)), warmup, stream, world), world)
        out[transport] = (us, lat, len(ring))
    del ring
    return out


def bench_gqa_decode(steps: int, warmup: int):
    """Grouped-head decode on one GPU: B=1, 32 query heads over 8 K/V heads,
    32768 tokens, D=128, fp16 and fp8 (e4m3) caches (both on the tensor-core
    kernel); then the ragged batch of the decode_ragged leg (B=8,
    lengths U[4096, 131072]) with 32 query heads over 8 K/V heads, fp16.
    Returns {case: (us, K/V bytes read)}."""
    import torch
    from pallas_flash.kernels import decoding as dec

    B, H, H_kv, N, D = 1, 32, 8, 32768, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(5000)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.float16)
    k = torch.randn((B, H_kv, N, D), device="cuda", generator=g)
    v = torch.randn((B, H_kv, N, D), device="cuda", generator=g)
    flush = L2Flush()
    stream = torch.cuda.current_stream()
    out = {}
    caches = {"f16": (k.half(), v.half(), 1.0, 1.0)}
    fp8 = getattr(torch, "float8_e4m3fn", None)
    if fp8 is not None:
        caches["fp8_e4m3"] = ((k / 0.25).to(fp8), (v / 0.25).to(fp8), 0.25, 0.25)
    for name, (kc, vc, ks, vs) in caches.items():
        def step():
            return dec.pallas_flash_decoding(q, kc, vc, k_scale=ks, v_scale=vs)
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        lat = _timed(step, steps, flush, stream)
        nbytes = 2 * kc.numel() * kc.element_size()
        ring = [(kc, vc)] + [(kc.clone(), vc.clone()) for _ in range(_copies(nbytes) - 1)]
        us = _steady(lambda kv: dec.pallas_flash_decoding(q, kv[0], kv[1], k_scale=ks, v_scale=vs),
                     ring, steps, warmup, stream)
        out[name] = (us, nbytes, lat, len(ring))
        del ring
    del caches, k, v
    # ragged batch, grouped heads
    Bg, Ng = RAG_B, RAG_NCAP
    lens = ragged_lens()
    qg = torch.randn((Bg, H, 1, D), device="cuda", generator=g).to(torch.float16)
    kg = torch.randn((Bg, H_kv, Ng, D), device="cuda", generator=g).to(torch.float16)
    vg = torch.randn((Bg, H_kv, Ng, D), device="cuda", generator=g).to(torch.float16)
    lens_d = torch.tensor(lens, dtype=torch.int32, device="cuda")

    def step_r():
        return dec.pallas_flash_decoding(qg, kg, vg, kv_lens=lens_d)
    for _ in range(warmup):
        step_r()
    torch.cuda.synchronize()
    lat = _timed(step_r, steps, flush, stream)
    us = _steady(lambda _: step_r(), [None], steps, warmup, stream)   # 2.5 GB of K/V: no copies needed
    out["ragged_f16"] = (us, 2 * int(sum(lens)) * H_kv * D * 2, lat, 1)
    return out


def profile_gqa(steps: int, warmup: int) -> float:
    """The fp16 case of the grouped-head leg alone (B=1, H=32 over 8 K/V
    heads, 32768 tokens), for ncu captures."""
    import torch
    from pallas_flash.kernels import decoding as dec

    B, H, H_kv, N, D = 1, 32, 8, 32768, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(5000)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.float16)
    k = torch.randn((B, H_kv, N, D), device="cuda", generator=g).to(torch.float16)
    v = torch.randn((B, H_kv, N, D), device="cuda", generator=g).to(torch.float16)
    flush = L2Flush()

    def step():
        return dec.pallas_flash_decoding(q, k, v)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    return _timed(step, steps, flush, torch.cuda.current_stream())


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["pu", "reference"], default="pu")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--profile-leg", choices=["attn", "decode", "gqa", "outproj"], default=None,
                    help="run only this leg and print no JSON (small runs for ncu captures)")
    ap.add_argument("--profile-batch", type=int, default=B,
                    help="batch of the attention profile leg (default: the bench workload's)")
    args = ap.parse_args()
    warmup = max(3, args.warmup)
    peaks = load_peaks()

    if args.impl == "reference":
        return run_reference(args, warmup)

    import torch
    rank, world, local = dist_init()
    if args.profile_leg == "decode":
        us = bench_decode(args.steps, warmup, rank, world, "peer")[0]
        print(f"decode leg: {us:.1f} us/step", flush=True)
        return
    if args.profile_leg == "gqa":
        us = profile_gqa(args.steps, warmup)
        print(f"grouped-head decode leg: {us:.1f} us/step", flush=True)
        return
    if args.profile_leg == "outproj":
        op = bench_outproj(args.steps, warmup, rank, world)
        print(f"out-projection leg: {op['peer'][0]:.1f} us/step", flush=True)
        return
    parity = run_parity(rank, world) if args.profile_leg is None else None
    clocks = ClockSampler(local).start()
    total_ms, fwd_ms, bwd_ms = bench_attention(args.steps, warmup, rank, world, clocks,
                                               batch=args.profile_batch if args.profile_leg else B)
    clk = clocks.stop()
    if args.profile_leg == "attn":
        print(f"attention leg: {total_ms / args.steps:.3f} ms/step", flush=True)
        return
    ms_step = allreduce_max(total_ms / args.steps, world)
    value = STEP_FLOPS * world / (ms_step * 1e-3) / 1e12
    bwd_ms_max = allreduce_max(bwd_ms, world)
    fwd_ms_max = allreduce_max(fwd_ms, world)
    e2e_dt, h2d, d2h = bench_attention_e2e(max(1, args.e2e_steps), 1, rank, world)
    dec_steps = max(5, min(args.steps, 50))
    dec_us, dec_kus, dec_bytes, dec_steady, dec_copies = bench_decode(dec_steps, warmup, rank, world, "peer")
    nccl = bench_decode(dec_steps, warmup, rank, world, "nccl") if world > 1 else None
    rag_us, rag_paged_us, rag_contig_us, rag_bytes = bench_ragged_decode(max(5, min(args.steps, 20)),
                                                                         warmup, rank, world)
    gqa = bench_gqa_decode(max(5, min(args.steps, 50)), warmup) if world == 1 else None
    c1 = bench_c1(max(10, min(args.steps, 50)), warmup) if world == 1 else None
    long_ms = bench_attention_long(max(3, min(args.steps, 5)), warmup) if world == 1 else None
    op = bench_outproj(max(5, min(args.steps, 20)), warmup, rank, world)

    if rank == 0:
        bwd_flops = FWD_FLOPS * 2.5
        achieved = bwd_flops / (bwd_ms_max * 1e-3) / 1e12
        roof = {"kernel": "attn_bwd (prep + fused dK/dV/dQ + dQ conversion kernels, one pu_attn_bwd call)",
                "bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                "peak_source": peaks["source"] + " bf16 burst",
                "traffic": NCU_TRAFFIC_BYTES["attn_bwd"],
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch: "
                                  + TRAFFIC_CAPTURE}
        fwd_ach = FWD_FLOPS / (fwd_ms_max * 1e-3) / 1e12
        cpu = None
        if world == 1:
            cv, cdt, sample = cpu_attention_sample()
            cpu = {"value": round(cv, 4), "unit": "TFLOP/s", "cores": cpu_threads(), "kind": "port",
                   "sample": sample + f" ({cdt:.1f} s)"}
        dec_total_bytes = dec_bytes * world
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic N(0,1) bf16 inputs generated on device (seeded)",
            "config": {"workload": "causal flash-attention fwd+bwd, B=4 H=16 N=4096 D=128 bf16 per GPU "
                                   "(heads partitioned across GPUs, no collective)",
                       "global_batch": B, "seq_len": N, "heads_per_gpu": H, "global_heads": H * world,
                       "head_dim": D, "parallelism": f"heads{world}",
                       "l2": "inputs 268 MB per GPU > 126 MB L2 (no flush needed)"},
            "roofline": roof,
            "roofline_fwd": {"kernel": "attn_fwd", "achieved": round(fwd_ach, 1),
                             "frac": round(fwd_ach / peaks["bf16_tflops"], 4), "unit": "TFLOP/s",
                             "traffic": NCU_TRAFFIC_BYTES["attn_fwd"]},
            "cpu_baseline": cpu,
            "e2e": {"value": round(STEP_FLOPS * world / e2e_dt / 1e12, 3), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_dt * 1e3, 3),
                    "path": "pallas_flash_attention(host pinned q,k,v) + autograd backward"},
            "gpu_launches": 4 * args.steps,
            "clocks": clk,
            "decode": {"workload": f"split-KV decode B=1 H=32 N=32768 D=128 fp16 cache, sequence-sharded over {world} GPU(s)"
                                   + (", (m,l,o) records stored into every rank's exchange buffer over "
                                      "NVLink + bounded-wait flag merge (no collective)" if world > 1 else ""),
                       "us_per_step": round(dec_steady, 2),
                       "GB_s": round(dec_total_bytes / (dec_steady * 1e-6) / 1e9, 1),
                       "frac_aggregate_hbm": round(dec_total_bytes / (dec_steady * 1e-6) / 1e9 /
                                                   (peaks["hbm_gbs"] * world), 4),
                       "timing": f"{dec_steps} steps back to back over {dec_copies} cache copies "
                                 "(each step's shard out of L2), one pair of CUDA events, the host "
                                 "ahead of the device (steps enqueued before the first event fires)",
                       "latency_us": round(dec_us, 2),
                       "latency_timing": "one step between CUDA events after a 1 GiB L2 flush, median "
                                         "(includes ~6-7 us of launch gap: a one-element kernel reads "
                                         "6.9 us this way)",
                       "kernel_us": round(dec_kus, 2),
                       "kernel_timing": "the local split-KV kernel alone, back to back over the same copies",
                       "nccl_allgather_us_per_step": round(nccl[3], 2) if nccl else None,
                       "nccl_allgather_latency_us": round(nccl[0], 2) if nccl else None,
                       "roofline": {"bound": "hbm", "achieved": round(dec_bytes / (dec_kus * 1e-6) / 1e9, 1),
                                    "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                    "frac": round(dec_bytes / (dec_kus * 1e-6) / 1e9 / peaks["hbm_gbs"], 4),
                                    "traffic": NCU_TRAFFIC_BYTES["split_kv"] if world == 1 else None},
                       "l2": "us_per_step and kernel_us: each step's cache copy is out of L2 (copies "
                             "x shard > 2 x L2); latency_us: 1 GiB written, then 1 GiB read, before the step"},
        }
        hbm = peaks["hbm_gbs"]
        line["decode_ragged"] = {
            "workload": f"ragged split-KV decode B={RAG_B} H={RAG_H} D={RAG_D} fp16, lengths "
                        f"U[4096,{RAG_NCAP}] rounded to 128 (seeded), dense cache padded to "
                        f"{RAG_NCAP}, sequence-sharded over {world} GPU(s)",
            "algorithmic_bytes": rag_bytes,
            "dense": {"us_per_step": round(rag_us, 2),
                      "GB_s": round(rag_bytes / (rag_us * 1e-6) / 1e9, 1),
                      "frac": round(rag_bytes / (rag_us * 1e-6) / 1e9 / (hbm * world), 4),
                      "sharding": "by held tokens (length_balanced_split)" if world > 1 else "one GPU"},
            "l2": "1 GiB buffer written, then another 1 GiB read, before every step"}
        op_flops = 2 * OP_T * OP_K * OP_N
        link_bytes = 2 * (world - 1) * OP_T * OP_N * 2 // world   # partials out + results out, per rank
        op_floor_us = max(op_flops / (peaks["bf16_tflops"] * 1e12), link_bytes / 770e9) * 1e6
        line["outproj"] = {
            "workload": f"out-projection + TP all-reduce: per rank [{OP_T}, {OP_K}] x [{OP_K}, {OP_N}] bf16, "
                        f"partials summed over {world} GPU(s), result on every rank",
            "timing": f"*_us: calls back to back over {op['peer'][2]} copies of the activation (out of "
                      "L2), one pair of CUDA events; *_latency_us: median single call started on an "
                      "idle GPU (includes the host-side work before the launch)",
            "fused_peer_us": round(op["peer"][0], 2),
            ("matmul_nccl_allreduce_us" if world > 1 else "cublas_matmul_us"): round(op["nccl"][0], 2),
            "fused_peer_latency_us": round(op["peer"][1], 2),
            ("matmul_nccl_allreduce_latency_us" if world > 1 else "cublas_matmul_latency_us"):
                round(op["nccl"][1], 2),
            "gemm_TFLOP_s_per_gpu": round(op_flops / (op["peer"][0] * 1e-6) / 1e12, 1),
            "nvlink_bytes_out_per_gpu": link_bytes,
            "roofline": {"bound": "tensor" if world == 1 else "max(tensor, nvlink)",
                         "floor_us": round(op_floor_us, 2),
                         "frac": round(op_floor_us / op["peer"][0], 4),
                         "peaks": f"{peaks['bf16_tflops']} TFLOP/s bf16 (measured), 770 GB/s NVLink per "
                                  "direction (measured peer copy)"}}
        if long_ms:
            lf, lb = long_ms
            line["attn_long"] = {
                "workload": f"non-causal fwd+bwd B={LONG_B} H={LONG_H} N={LONG_N} D={D} bf16, "
                            "Q/K/V ~ N(0,0.5), dO ~ N(0,1), one GPU",
                "fwd_ms": round(lf, 3), "bwd_ms": round(lb, 3),
                "TFLOP_s": round(LONG_FWD_FLOPS * 3.5 / ((lf + lb) * 1e-3) / 1e12, 1),
                "fwd_TFLOP_s": round(LONG_FWD_FLOPS / (lf * 1e-3) / 1e12, 1),
                "bwd_TFLOP_s": round(LONG_FWD_FLOPS * 2.5 / (lb * 1e-3) / 1e12, 1),
                "frac": round(LONG_FWD_FLOPS * 3.5 / ((lf + lb) * 1e-3) / 1e12 / peaks["bf16_tflops"], 4)}
        if gqa:
            line["decode_gqa"] = {
                "workload": "grouped-head decode B=1 H=32 H_kv=8 N=32768 D=128, one GPU (f16: "
                            "gqa_tc_kernel, tcgen05 kind::f16 K-tile x query-group; fp8_e4m3: the "
                            "same kernel with kind::f8f6f4 products on the e4m3 tiles); ragged_f16: "
                            "B=8 H=32 H_kv=8 D=128 with the decode_ragged lengths",
                "l2": "us_per_step: steps back to back over enough cache copies that each step's "
                      "cache is out of L2; latency_us: one step after a 1 GiB L2 flush"}
            for name, (us, nbytes, lat, ncopies) in gqa.items():
                line["decode_gqa"][name] = {
                    "us_per_step": round(us, 2), "kv_bytes": nbytes,
                    "GB_s": round(nbytes / (us * 1e-6) / 1e9, 1),
                    "frac": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4),
                    "timing": f"back to back over {ncopies} cache copies",
                    "latency_us": round(lat, 2)}
        if rag_contig_us is not None:
            line["decode_ragged"]["dense_contiguous_chunks"] = {
                "us_per_step": round(rag_contig_us, 2),
                "GB_s": round(rag_bytes / (rag_contig_us * 1e-6) / 1e9, 1),
                "frac": round(rag_bytes / (rag_contig_us * 1e-6) / 1e9 / (hbm * world), 4),
                "sharding": "rank r holds positions [r*N/G, (r+1)*N/G) of the padded capacity"}
        if c1 is not None:
            c1_us, c1_lat, c1_copies = c1
            c1_cpu_s = cpu_c1_sample()
            line["attn_c1"] = {
                "workload": f"causal forward B={C1_B} H={C1_H} N={C1_N} D={D} bf16 (the reference's "
                            "CPU baseline_mha configuration), one GPU",
                "timing": f"calls back to back over {c1_copies} copies of q, k, v (out of L2); "
                          "latency_us: one call after a 1 GiB L2 flush",
                "latency_us": round(c1_lat, 2),
                "us_per_call": round(c1_us, 2),
                "TFLOP_s": round(C1_FLOPS / (c1_us * 1e-6) / 1e12, 1),
                "frac": round(C1_FLOPS / (c1_us * 1e-6) / 1e12 / peaks["bf16_tflops"], 4),
                "cpu_baseline": {"value": round(c1_cpu_s * 1e6, 1), "unit": "us/call",
                                 "cores": cpu_threads(), "kind": "port",
                                 "sample": "whole workload, oracle causal baseline_mha restatement, "
                                           "numpy fp32, best of 3"}}
        line["parity"] = parity
        if rag_paged_us is not None:
            line["decode_ragged"]["paged"] = {
                "page_size": RAG_PAGE, "page_order": "shuffled",
                "us_per_step": round(rag_paged_us, 2),
                "GB_s": round(rag_bytes / (rag_paged_us * 1e-6) / 1e9, 1),
                "frac": round(rag_bytes / (rag_paged_us * 1e-6) / 1e9 / hbm, 4)}
        if world == 1:
            dus, dsample = cpu_decode_sample()
            line["decode"]["cpu_baseline"] = {"value": round(dus, 1), "unit": "us/step",
                                              "cores": cpu_threads(), "kind": "port", "sample": dsample}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        from pallas_flash.distributed import peer
        peer.close_all()
        dist.barrier()
        dist.destroy_process_group()
    else:
        import torch.distributed as dist
        if dist.is_initialized():
            from pallas_flash.distributed import peer
            peer.close_all()
            dist.destroy_process_group()
    if parity is not None and not all(v["ok"] for v in parity.values()):
        bad = [k for k, v in parity.items() if not v["ok"]]
        print(f"parity miss: {bad}", file=sys.stderr, flush=True)
        sys.exit(1)


def run_reference(args, warmup):
    """The reference algorithm on host CPU cores (numpy port of its pure-JAX
    path; JAX is not installed).  Rank 0 only.  Each step is a bounded sample:
    the fwd+bwd of one of the 64 (b, h) heads of a GPU's workload; the line
    reports that sample's measured time and the throughput it implies."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    vals, times = [], []
    sample = ""
    for i in range(warmup + args.steps):
        v, dt, sample = cpu_attention_sample(heads=1)
        if i >= warmup:
            vals.append(v)
            times.append(dt)
    value = statistics.median(vals)
    sample_ms = statistics.median(times) * 1e3
    heads = B * H
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": warmup, "ms_per_step": round(sample_ms, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1) inputs (seeded numpy PCG64)",
        "config": {"workload": "causal flash-attention fwd+bwd, B=4 H=16 N=4096 D=128 per GPU",
                   "global_batch": B, "seq_len": N, "heads_per_gpu": H, "head_dim": D,
                   "parallelism": f"heads{world}"},
        "sample": {"heads_per_step": 1, "of_heads": heads, "measured_ms_per_step": round(sample_ms, 1),
                   "extrapolated_full_step_ms": round(sample_ms * heads, 1),
                   "note": "ms_per_step is the measured one-head sample; value is its FLOPs / time "
                           "(the whole workload would take extrapolated_full_step_ms on this host)"},
        "cpu_baseline": {"value": round(value, 4), "kind": "port", "cores": cpu_threads(),
                         "sample": sample + " per step; JAX reference not installable here, so the "
                                            "numpy restatement in oracle/ stands in"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
