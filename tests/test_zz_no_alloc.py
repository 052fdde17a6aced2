"""The allocation-free decode entry point, pu_decode_noalloc.

Some callers cannot hand the library device scratch memory (a custom-call
handler that only receives its operands and results, or a runtime that plans
all device memory up front and forbids later allocation).  For them the
library keeps a fixed 8 MiB scratch array in its own device memory.  These
tests call the entry point through the C ABI (ctypes) and check that two
calls in a row give what the workspace-taking pu_decode gives and what the
CPU oracle's decode (oracle/attention.py, the restatement of the
reference's decode step) gives, within the bf16 output tolerance used by the
other decode tests, and that problems too large for the fixed scratch are
refused before anything runs.

This file is collected last on purpose, and it passes both on its own in a
fresh process and after the rest of the suite.
"""
from __future__ import annotations

import math

import pytest
import torch

from helpers import assert_close_lse, assert_close_o, randn, to_np
from oracle import attention as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(built_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from pallas_flash import _lib
    return _lib


def _with_workspace(lib, q, k, v, lens):
    B, H, n, D = k.shape
    o = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((B, H), dtype=torch.float32, device="cuda")
    need = int(lib.lib().pu_decode_workspace_size(B, H, n, D))
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    lib.check(lib.lib().pu_decode(q.data_ptr(), lib.PU_DTYPE_F16, k.data_ptr(), v.data_ptr(),
                                  lib.PU_DTYPE_F16, lens.data_ptr() if lens is not None else None,
                                  o.data_ptr(), lse.data_ptr(), ws.data_ptr(), need, B, H, n, D,
                                  1.0 / math.sqrt(D), stream), "pu_decode")
    return o, lse


def _no_alloc(lib, q, k, v, lens):
    B, H, n, D = k.shape
    o = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((B, H), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    lib.check(lib.lib().pu_decode_noalloc(q.data_ptr(), lib.PU_DTYPE_F16, k.data_ptr(),
                                          v.data_ptr(), lib.PU_DTYPE_F16,
                                          lens.data_ptr() if lens is not None else None,
                                          o.data_ptr(), lse.data_ptr(), B, H, n, D,
                                          1.0 / math.sqrt(D), stream), "pu_decode_noalloc")
    return o, lse


@pytest.mark.parametrize("B,H,n,ragged", [(1, 32, 32768, False), (3, 4, 5000, True)])
def test_no_alloc_matches_workspace_entry_point(lib, B, H, n, ragged):
    D = 128
    q = randn((B, H, 1, D), 61, dtype=torch.float16).cuda()
    k = randn((B, H, n, D), 62, dtype=torch.float16).cuda()
    v = randn((B, H, n, D), 63, dtype=torch.float16).cuda()
    lens = None
    if ragged:
        lens = torch.tensor([n, 1, n // 3][:B], dtype=torch.int32, device="cuda")
    ref_o, ref_lse = _with_workspace(lib, q, k, v, lens)
    orc_o, orc_lse = orc.decode_forward(to_np(q), to_np(k), to_np(v),
                                        kv_lens=None if lens is None else lens.cpu().numpy())
    for _ in range(2):  # two calls in a row share (and must re-clear) the static scratch
        o, lse = _no_alloc(lib, q, k, v, lens)
        torch.cuda.synchronize()
        assert lib.device_status()[0] == 0
        assert_close_o(to_np(o), to_np(ref_o))
        assert_close_lse(to_np(lse), to_np(ref_lse))
        assert_close_o(to_np(o), orc_o, what="o vs oracle")
        assert_close_lse(to_np(lse).reshape(orc_lse.shape), orc_lse)


def test_no_alloc_rejects_problems_beyond_the_scratch(lib):
    D = 128
    q = torch.zeros((1, 1, 1, D), dtype=torch.float16, device="cuda")
    k = torch.zeros((1, 1, 16, D), dtype=torch.float16, device="cuda")
    o = torch.empty((1, 1, 1, D), dtype=torch.bfloat16, device="cuda")
    # B*H = 20000 (h) x 1 split x 130 floats needs ~10.4 MB > 8 MiB: refused on the host
    rc = lib.lib().pu_decode_noalloc(q.data_ptr(), lib.PU_DTYPE_F16, k.data_ptr(), k.data_ptr(),
                                     lib.PU_DTYPE_F16, None, o.data_ptr(), None, 1, 20000, 16, D,
                                     0.1, torch.cuda.current_stream().cuda_stream)
    assert rc == lib.PU_ERR_WORKSPACE
    assert b"static scratch" in lib.lib().pu_last_error()
