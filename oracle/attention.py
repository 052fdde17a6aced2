"""CPU oracle for the attention hot path — TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module.  It is used by `tests/`, by
`__graft_entry__.smoke()` (as the checker) and by `bench.py`'s CPU-baseline
leg.  It restates, in numpy, the arithmetic of the reference project
(ArjunSom9/Pallas-Unbound, a JAX/Pallas TPU code base) for the hot path:

  * `mha_forward`        — softmax(q k^T * scale [+ causal mask]) v and its
                           LogSumExp, computed in fp32/fp64 from the exact
                           bf16/fp16 input values.  Restates
                           benchmarks/baseline_mha.py:22-58 (causal:
                           triu(-inf, k=1), lines 47-50) and the fp32
                           non-causal test reference
                           tests/test_correctness.py:22-33.
  * `mha_backward`       — dQ, dK, dV of the above (the closed form of the
                           autodiff of baseline_mha; the reference has no
                           backward kernel).
  * `pipeline_emulation` — the reference KERNEL's blockwise arithmetic:
                           128-row K/V blocks, fp32 m/l/o carries, P rounded
                           to bf16 before P.V, padded keys masked with -1e10.
                           Restates kernels/pipeline.py:14-60 with
                           low_level/intrinsics.py:11-37.
  * `decode_forward`     — one query token against a KV cache, optional
                           per-sequence lengths.  Restates
                           benchmarks/inference_decode.py:32-44 and
                           kernels/decoding.py:19-60 (mask past the length,
                           decoding.py:42-44).
  * `decode_partial` / `lse_combine` — per-shard (m, l, o) partials and their
                           stable LogSumExp merge: the online-softmax update
                           of pipeline.py:47-52 applied across shards, which
                           is what the reference documents for split-KV
                           decode (README.md:41-46) but never implements.
  * `paged_to_dense` / `paged_append` — the paged KV cache (page pool +
                           page table) the paged decode and append kernels
                           use; no reference counterpart (the reference's
                           decode reads a dense cache, decoding.py:86-103),
                           so these define the layout the kernels are
                           checked against.

Parity pinning: the reference cannot run in this environment (it needs JAX
and a TPU; JAX is not installed), so no reference outputs exist to compare
against.  The oracle is pinned to the reference's own known-answer tests
(tests/test_numerics.py:29-117: uniform logits give O == V, zero / very
negative inputs stay finite, bf16 output) and to analytic identities of the
algorithm; see tests/test_oracle.py.
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634

# ---------------------------------------------------------------------------
# dtype helpers (bf16 has no numpy dtype; values are carried as float32)
# ---------------------------------------------------------------------------


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    nan = np.isnan(a)
    out[nan] = np.nan
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 values that are exactly bf16 -> their uint16 bit patterns."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# training attention
# ---------------------------------------------------------------------------


def _scores(qh: np.ndarray, kh: np.ndarray, scale: float, causal: bool, dtype) -> np.ndarray:
    s = (qh.astype(dtype) @ kh.astype(dtype).T) * dtype(scale)
    if causal:
        nq, nk = s.shape
        # baseline_mha.py:48-49: triu(full(-inf), k=1) added to the logits
        mask = np.triu(np.ones((nq, nk), dtype=bool), k=1)
        s = np.where(mask, -np.inf, s)
    return s


def mha_forward(q, k, v, *, causal: bool, scale: float | None = None, dtype=np.float64,
                row_chunk: int = 4096):
    """Exact attention.  q [B,H,Nq,D], k/v [B,H,Nkv,D] -> (o [B,H,Nq,D], lse [B,H,Nq]).

    Computed per (b, h) and per block of `row_chunk` query rows so large
    sequences stay within memory; `dtype` is the accumulation type.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    B, H, Nq, D = q.shape
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    o = np.empty((B, H, Nq, D), dtype=dtype)
    lse = np.empty((B, H, Nq), dtype=dtype)
    for b in range(B):
        for h in range(H):
            kh = k[b, h].astype(dtype)
            vh = v[b, h].astype(dtype)
            for r0 in range(0, Nq, row_chunk):
                r1 = min(Nq, r0 + row_chunk)
                s = (q[b, h, r0:r1].astype(dtype) @ kh.T) * dtype(scale)
                if causal:
                    rows = np.arange(r0, r1)[:, None]
                    cols = np.arange(s.shape[1])[None, :]
                    s = np.where(cols > rows, -np.inf, s)
                m = s.max(axis=1, keepdims=True)
                p = np.exp(s - m)
                l = p.sum(axis=1, keepdims=True)
                o[b, h, r0:r1] = (p @ vh) / l
                lse[b, h, r0:r1] = (m + np.log(l))[:, 0]
    return o, lse


def mha_backward(q, k, v, o, lse, do, *, causal: bool, scale: float | None = None,
                 dtype=np.float64, row_chunk: int = 4096):
    """Gradients of mha_forward w.r.t. q, k, v for upstream gradient `do`.

    P = exp(S - lse); dV = P^T dO; dP = dO V^T; Delta = rowsum(dO * O);
    dS = P * (dP - Delta); dQ = scale dS K; dK = scale dS^T Q.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    B, H, Nq, D = q.shape
    Nkv = k.shape[2]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    dq = np.zeros((B, H, Nq, D), dtype=dtype)
    dk = np.zeros((B, H, Nkv, D), dtype=dtype)
    dv = np.zeros((B, H, Nkv, D), dtype=dtype)
    for b in range(B):
        for h in range(H):
            kh = k[b, h].astype(dtype)
            vh = v[b, h].astype(dtype)
            for r0 in range(0, Nq, row_chunk):
                r1 = min(Nq, r0 + row_chunk)
                qh = q[b, h, r0:r1].astype(dtype)
                doh = np.asarray(do[b, h, r0:r1], dtype=np.float32).astype(dtype)
                oh = np.asarray(o[b, h, r0:r1]).astype(dtype)
                s = (qh @ kh.T) * dtype(scale)
                if causal:
                    rows = np.arange(r0, r1)[:, None]
                    cols = np.arange(Nkv)[None, :]
                    s = np.where(cols > rows, -np.inf, s)
                p = np.exp(s - np.asarray(lse[b, h, r0:r1], dtype=dtype)[:, None])
                dv[b, h] += p.T @ doh
                dp = doh @ vh.T
                delta = (doh * oh).sum(axis=1, keepdims=True)
                ds = p * (dp - delta)
                dq[b, h, r0:r1] = dtype(scale) * (ds @ kh)
                dk[b, h] += dtype(scale) * (ds.T @ qh)
    return dq, dk, dv


def pipeline_emulation(q, k, v, *, causal: bool = False, scale: float | None = None,
                       block_kv: int = 128, original_seq_len: int | None = None):
    """The reference kernel's arithmetic for one call (pipeline.py:14-60).

    fp32 accumulators o, m = -inf, l = 0; per 128-row K/V block:
    S = Q K^T (fp32), keys at or past `original_seq_len` set to -1e10,
    m' = max(m, rowmax S), P = bf16(exp(S - m')), l' = l e^{m-m'} + sum P,
    o' = o e^{m-m'} + P V.  Returns (o / l, m, l) like pipeline_kv_loop; the
    scale is applied to S here instead of being folded into bf16 q
    (interface.py:43-44), and `causal` adds the baseline_mha mask that the
    reference kernel lacks.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    B, H, Nq, D = q.shape
    Nkv = k.shape[2]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    if original_seq_len is None:
        original_seq_len = Nkv
    o_out = np.empty((B, H, Nq, D), dtype=np.float32)
    m_out = np.empty((B, H, Nq), dtype=np.float32)
    l_out = np.empty((B, H, Nq), dtype=np.float32)
    n_steps = (Nkv + block_kv - 1) // block_kv
    rows = np.arange(Nq)[:, None]
    for b in range(B):
        for h in range(H):
            o_acc = np.zeros((Nq, D), dtype=np.float32)
            m_i = np.full((Nq, 1), -np.inf, dtype=np.float32)
            l_i = np.zeros((Nq, 1), dtype=np.float32)
            for j in range(n_steps):
                sl = slice(j * block_kv, min(Nkv, (j + 1) * block_kv))
                kb = k[b, h, sl]
                vb = v[b, h, sl]
                s = (q[b, h] @ kb.T).astype(np.float32) * np.float32(scale)
                cols = np.arange(sl.start, sl.stop)[None, :]
                s = np.where(cols < original_seq_len, s, np.float32(-1e10))
                if causal:
                    s = np.where(cols > rows, np.float32(-np.inf), s)
                m_new = np.maximum(m_i, s.max(axis=1, keepdims=True))
                p = bf16_round(np.exp(s - m_new).astype(np.float32))
                with np.errstate(invalid="ignore"):
                    alpha = np.exp(m_i - m_new).astype(np.float32)
                alpha = np.where(np.isnan(alpha), np.float32(0.0), alpha)
                l_i = l_i * alpha + p.sum(axis=1, keepdims=True)
                o_acc = o_acc * alpha + p @ vb
                m_i = m_new
            o_out[b, h] = o_acc / l_i
            m_out[b, h] = m_i[:, 0]
            l_out[b, h] = l_i[:, 0]
    return o_out, m_out, l_out


# ---------------------------------------------------------------------------
# decode
# ---------------------------------------------------------------------------


def decode_forward(q, k_cache, v_cache, *, kv_lens=None, scale: float | None = None,
                   dtype=np.float64):
    """One query token per (b, h).  q [B,H,1,D], caches [B,H_kv,N,D]; returns (o [B,H,1,D], lse [B,H]).

    inference_decode.py:32-44 (softmax(q K^T / sqrt(D)) V) with the
    length mask of decoding.py:42-44 when kv_lens is given.  With
    H_kv < H (grouped heads, no reference counterpart) query head h reads
    K/V head h // (H // H_kv).
    """
    q = np.asarray(q, dtype=np.float32)
    B, H, _, D = q.shape
    N = k_cache.shape[2]
    G = H // k_cache.shape[1]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    o = np.zeros((B, H, 1, D), dtype=dtype)
    lse = np.full((B, H), -np.inf, dtype=dtype)
    for b in range(B):
        n = N if kv_lens is None else int(min(N, kv_lens[b]))
        if n <= 0:
            continue
        for h in range(H):
            kh = np.asarray(k_cache[b, h // G, :n], dtype=np.float32).astype(dtype)
            vh = np.asarray(v_cache[b, h // G, :n], dtype=np.float32).astype(dtype)
            s = (kh @ q[b, h, 0].astype(dtype)) * dtype(scale)
            m = s.max()
            p = np.exp(s - m)
            l = p.sum()
            o[b, h, 0] = (p @ vh) / l
            lse[b, h] = m + np.log(l)
    return o, lse


def decode_partial(q, k_shard, v_shard, *, kv_offset: int, kv_lens=None,
                   scale: float | None = None, dtype=np.float64):
    """(m, l, o) of one sequence shard: m = max logit, l = sum e^{s-m}, o = sum e^{s-m} v.

    Empty shards (all positions past the length) give m = -inf, l = 0, o = 0.
    Returns a packed float array [B*H, D+2] = {m, l, o[D]}.
    """
    q = np.asarray(q, dtype=np.float32)
    B, H, _, D = q.shape
    n_local = k_shard.shape[2]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    out = np.zeros((B * H, D + 2), dtype=dtype)
    out[:, 0] = -np.inf
    for b in range(B):
        total = kv_offset + n_local if kv_lens is None else int(kv_lens[b])
        n = max(0, min(n_local, total - kv_offset))
        if n == 0:
            continue
        for h in range(H):
            kh = np.asarray(k_shard[b, h, :n], dtype=np.float32).astype(dtype)
            vh = np.asarray(v_shard[b, h, :n], dtype=np.float32).astype(dtype)
            s = (kh @ q[b, h, 0].astype(dtype)) * dtype(scale)
            m = s.max()
            p = np.exp(s - m)
            r = out[b * H + h]
            r[0] = m
            r[1] = p.sum()
            r[2:] = p @ vh
    return out


def paged_to_dense(pool, page_table, kv_lens, page_size: int, n: int | None = None):
    """Gather a paged cache pool [P, H, page_size, D] into a dense [B, H, n, D] cache.

    Token t of sequence b is row t % page_size of page page_table[b, t // page_size];
    positions at or past kv_lens[b] are left zero.  The reference has no
    paged cache (its decode reads a dense [B,H,N,D] cache, decoding.py:86-103):
    this is the definition the paged kernels are checked against.
    """
    pool = np.asarray(pool)
    table = np.asarray(page_table)
    B = table.shape[0]
    _, H, ps, D = pool.shape
    assert ps == page_size
    if n is None:
        n = table.shape[1] * page_size
    out = np.zeros((B, H, n, D), dtype=pool.dtype)
    for b in range(B):
        L = int(kv_lens[b])
        for t0 in range(0, L, page_size):
            rows = min(page_size, L - t0)
            out[b, :, t0:t0 + rows] = pool[table[b, t0 // page_size], :, :rows]
    return out


def paged_append(k_pool, v_pool, page_table, kv_lens, k_new, v_new, page_size: int):
    """In-place append of one token per sequence; returns the new lengths.

    Sequences whose next position has no valid page (past the table, or an
    entry outside [0, P)) are left unchanged, as the append kernel does.
    """
    table = np.asarray(page_table)
    lens = np.array(kv_lens, dtype=np.int64)
    P = k_pool.shape[0]
    for b in range(table.shape[0]):
        pos = int(lens[b])
        slot = pos // page_size
        if pos < 0 or slot >= table.shape[1]:
            continue
        pg = int(table[b, slot])
        if not 0 <= pg < P:
            continue
        k_pool[pg, :, pos % page_size] = k_new[b, :, 0]
        v_pool[pg, :, pos % page_size] = v_new[b, :, 0]
        lens[b] = pos + 1
    return lens


def lse_combine(partials):
    """Merge G packed partials [G, BH, D+2] -> (o [BH, D], lse [BH]).

    M = max_g m_g; L = sum_g l_g e^{m_g - M}; O = sum_g o_g e^{m_g - M} / L.
    """
    parts = np.asarray(partials, dtype=np.float64)
    m = parts[:, :, 0]
    M = m.max(axis=0)
    with np.errstate(invalid="ignore"):
        w = np.where(np.isneginf(m), 0.0, np.exp(m - M[None, :]))
    L = (w * parts[:, :, 1]).sum(axis=0)
    O = (w[:, :, None] * parts[:, :, 2:]).sum(axis=0)
    with np.errstate(invalid="ignore", divide="ignore"):
        o = np.where(L[:, None] > 0, O / L[:, None], 0.0)
        lse = np.where(L > 0, M + np.log(np.where(L > 0, L, 1.0)), -np.inf)
    return o, lse


# ---------------------------------------------------------------------------
# tolerance checks (the bar the parity tests apply)
# ---------------------------------------------------------------------------


def compare(actual, expected):
    """Max-abs error, max |expected|, and norm-relative error ||a-e|| / ||e||."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    diff = np.abs(a - e)
    max_abs = float(diff.max()) if diff.size else 0.0
    ref_max = float(np.abs(e).max()) if e.size else 0.0
    denom = float(np.linalg.norm(e.ravel()))
    rel = float(np.linalg.norm((a - e).ravel()) / denom) if denom > 0 else float(np.linalg.norm(a.ravel()))
    return {"max_abs": max_abs, "ref_max": ref_max, "rel": rel}
