"""Generate the golden fixtures of the attention oracle (run from the repo root):

    python tests/golden/make_golden.py

The reference (JAX/Pallas) cannot run in this environment, so these fixtures
freeze the oracle's outputs on small seeded inputs (numpy PCG64): bf16
inputs stored as uint16 bit patterns, fp32/fp64 outputs.  tests/test_oracle.py
checks the oracle still reproduces them and the GPU tests can compare the
kernels against them without recomputing.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import attention as orc  # noqa: E402

OUT = Path(__file__).resolve().parent


def bf16_inputs(shape, seed, scale=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(scale)
    return orc.bf16_round(x)


def main():
    cases = {
        # name: (B, H, Nq, Nkv, D, causal, seed, scale)
        "causal_1x2x192x128": (1, 2, 192, 192, 128, True, 101, 1.0),
        "noncausal_1x2x160x64": (1, 2, 160, 160, 64, False, 202, 0.5),
        "ragged_1x1x130x200": (1, 1, 130, 200, 128, False, 303, 1.0),
    }
    for name, (B, H, Nq, Nkv, D, causal, seed, scale) in cases.items():
        q = bf16_inputs((B, H, Nq, D), seed, scale)
        k = bf16_inputs((B, H, Nkv, D), seed + 1, scale)
        v = bf16_inputs((B, H, Nkv, D), seed + 2, scale)
        do = bf16_inputs((B, H, Nq, D), seed + 3)
        o, lse = orc.mha_forward(q, k, v, causal=causal)
        dq, dk, dv = orc.mha_backward(q, k, v, o, lse, do, causal=causal)
        np.savez_compressed(
            OUT / f"attn_{name}.npz",
            q=orc.bf16_bits(q), k=orc.bf16_bits(k), v=orc.bf16_bits(v), do=orc.bf16_bits(do),
            causal=np.array(causal), o=o.astype(np.float32), lse=lse.astype(np.float32),
            dq=dq.astype(np.float32), dk=dk.astype(np.float32), dv=dv.astype(np.float32))
    # decode: fp16 cache with ragged lengths, and its 4-way sequence split
    rng = np.random.Generator(np.random.PCG64(404))
    B, H, N, D = 3, 2, 256, 128
    q = rng.standard_normal((B, H, 1, D), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((B, H, N, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((B, H, N, D), dtype=np.float32).astype(np.float16)
    lens = np.array([256, 77, 200], dtype=np.int32)
    o, lse = orc.decode_forward(q, k, v, kv_lens=lens)
    G = 4
    parts = np.stack([orc.decode_partial(q, k[:, :, g * N // G:(g + 1) * N // G],
                                         v[:, :, g * N // G:(g + 1) * N // G],
                                         kv_offset=g * N // G, kv_lens=lens) for g in range(G)])
    np.savez_compressed(OUT / "decode_3x2x256.npz", q=q, k=k, v=v, lens=lens,
                        o=o.astype(np.float32), lse=lse.astype(np.float32),
                        partials=parts.astype(np.float32))
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()
