"""Seeded input generation and tolerance checks shared by the tests."""
from __future__ import annotations

import numpy as np
import torch

from oracle import attention as orc

# Tolerances of the parity bar (bf16 outputs, fp32 LSE, gradients).
O_MAX_ABS = 2e-2
O_REL = 1e-2
LSE_ABS = 1e-3
GRAD_REL = 3e-2


def randn(shape, seed: int, scale: float = 1.0, dtype=torch.bfloat16) -> torch.Tensor:
    """N(0, scale^2) values from a numpy PCG64 stream, rounded to `dtype` (CPU tensor)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(scale)
    return torch.from_numpy(x).to(dtype)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def assert_close_o(actual, expected, max_abs=O_MAX_ABS, rel=O_REL, what="o"):
    r = orc.compare(actual, expected)
    assert r["max_abs"] <= max_abs and r["rel"] <= rel, f"{what}: {r}"
    return r


def assert_close_lse(actual, expected, tol=LSE_ABS):
    r = orc.compare(actual, expected)
    assert r["max_abs"] <= tol, f"lse: {r}"
    return r


def assert_close_grad(actual, expected, rel=GRAD_REL, what="grad"):
    r = orc.compare(actual, expected)
    assert r["rel"] <= rel, f"{what}: {r}"
    return r


def one_rank_init_method() -> str:
    """Rendezvous URL for a one-rank process group: a store file in a fresh
    temporary directory (no TCP port, so no collision with a port another
    process is still holding)."""
    import os
    import tempfile
    return "file://" + os.path.join(tempfile.mkdtemp(prefix="pu_pg_"), "store")
