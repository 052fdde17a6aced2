"""The C-ABI library builds for sm_100a, loads on a host without a GPU, and
exports every entry point declared in include/pu_attn.h (no compute calls)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "pu_attn.h").read_text()
    return re.findall(r"PU_API\s+[\w\s\*]+?\b(pu_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("pu_attn_fwd", "pu_attn_bwd", "pu_decode", "pu_decode_partial",
                     "pu_decode_combine", "pu_last_error", "pu_device_status"):
        assert required in names


def test_library_exports_every_declared_symbol(built_lib):
    lib = ctypes.CDLL(str(built_lib))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"missing exports: {missing}"


def test_python_binding_matches_header(built_lib):
    from pallas_flash import _lib
    assert set(_lib.SIGNATURES) == set(declared_symbols())
    handle = _lib.lib()
    assert b"sm_100a" in handle.pu_version()


def test_build_recipe_targets_sm100a_only():
    """The recipe compiles for sm_100a machine code only: one -gencode whose
    code= is sm_100a, so no PTX for another architecture is embedded."""
    from conftest import load_build_module
    flags = load_build_module().ARCH_FLAGS
    assert flags == ["-gencode", "arch=compute_100a,code=sm_100a"], flags


@pytest.mark.gpu
def test_loaded_kernels_are_sm100a(built_lib):
    """On a B200, the kernels the runtime loads report binary version 100."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from pallas_flash import _lib
    arch = ctypes.c_int(0)
    _lib.check(_lib.lib().pu_binary_arch(ctypes.byref(arch)), "pu_binary_arch")
    assert arch.value == 100


def test_argument_errors_are_reported_without_gpu(built_lib):
    """Bad arguments are rejected on the host before any CUDA call."""
    from pallas_flash import _lib
    lib = _lib.lib()
    rc = lib.pu_attn_fwd(None, None, None, None, None, 1, 1, 1, 1, 128, 0.1, 0, None)
    assert rc == _lib.PU_ERR_INVALID_ARGUMENT
    assert b"null" in lib.pu_last_error()
    rc = lib.pu_decode_combine(None, 1, None, None, 1, 1, 128, None)
    assert rc == _lib.PU_ERR_INVALID_ARGUMENT


def test_comm_argument_errors_without_gpu(built_lib):
    """The communicator entry points check their arguments before touching
    NCCL or the GPU; destroying a null communicator is a no-op."""
    import ctypes as ct
    from pallas_flash import _lib
    lib = _lib.lib()
    comm = ct.c_void_p()
    assert lib.pu_comm_init(None, 1, 0, ct.byref(comm)) == _lib.PU_ERR_INVALID_ARGUMENT
    uid = (ct.c_uint8 * _lib.PU_COMM_ID_BYTES)()
    assert lib.pu_comm_init(uid, 2, 2, ct.byref(comm)) == _lib.PU_ERR_INVALID_ARGUMENT
    assert lib.pu_allgather_partials(None, None, 1, 1, 128, None, None) == _lib.PU_ERR_INVALID_ARGUMENT
    assert lib.pu_comm_destroy(None) == _lib.PU_OK
