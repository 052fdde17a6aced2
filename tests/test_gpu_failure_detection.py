"""Failure detection on the GPU without a fault.

Every device-side wait of the kernels is bounded.  A self-test kernel waits
on an mbarrier that nothing completes, with a 20 ms bound: the wait runs
out, the kernel records PU_ERR_DEVICE_TIMEOUT in the device status word and
returns.  The host reads the status, and the same CUDA context keeps running
real work correctly afterwards.
"""
from __future__ import annotations

import time

import pytest
import torch

from helpers import assert_close_o, randn, to_np
from oracle import attention as orc

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(built_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from pallas_flash import _lib
    from pallas_flash.ops.interface import pallas_flash_attention
    lib = _lib.lib()
    assert _lib.device_status() == (_lib.PU_OK, 0)
    t0 = time.perf_counter()
    assert lib.pu_selftest_wait_timeout(20_000_000, torch.cuda.current_stream().cuda_stream) == 0
    code, site = _lib.device_status()
    elapsed = time.perf_counter() - t0
    assert code == _lib.PU_ERR_DEVICE_TIMEOUT and site == 901
    assert elapsed < 5.0
    assert _lib.device_status() == (_lib.PU_OK, 0)          # read-and-clear
    # the context is intact: real work still runs and is correct
    q = randn((1, 2, 256, 128), 91)
    o = pallas_flash_attention(q.cuda(), q.cuda(), q.cuda(), causal=True)
    ro, _ = orc.mha_forward(to_np(q), to_np(q), to_np(q), causal=True)
    assert_close_o(to_np(o), ro)
    assert _lib.device_status() == (_lib.PU_OK, 0)


def test_selftest_rejects_unbounded_request(built_lib):
    from pallas_flash import _lib
    lib = _lib.lib()
    assert lib.pu_selftest_wait_timeout(0, None) == _lib.PU_ERR_INVALID_ARGUMENT
    assert lib.pu_selftest_wait_timeout(10**12, None) == _lib.PU_ERR_INVALID_ARGUMENT
