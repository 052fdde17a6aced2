"""ctypes binding of libpu_attn.so — the C ABI declared in include/pu_attn.h.

This is the Python side of the drop-in boundary: every compute call of the
package goes through these symbols.  There is no fallback: if the library
is missing or cannot load, `lib()` raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PU_OK = 0
PU_ERR_INVALID_ARGUMENT = 1
PU_ERR_UNSUPPORTED = 2
PU_ERR_CUDA = 3
PU_ERR_WORKSPACE = 4
PU_ERR_DEVICE_TIMEOUT = 5

PU_DTYPE_BF16 = 0
PU_DTYPE_F16 = 1
PU_DTYPE_F32 = 2
PU_DTYPE_FP8_E4M3 = 3

PU_COMM_ID_BYTES = 128

_LIB_PATH = Path(__file__).resolve().parent / "_native" / "libpu_attn.so"

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_float = ctypes.c_float
_size_t = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/pu_attn.h
SIGNATURES = {
    "pu_version": (ctypes.c_char_p, []),
    "pu_last_error": (ctypes.c_char_p, []),
    "pu_device_status": (_int, [ctypes.POINTER(_int)]),
    "pu_binary_arch": (_int, [ctypes.POINTER(_int)]),
    "pu_selftest_wait_timeout": (_int, [ctypes.c_uint64, _c_void_p]),
    "pu_attn_fwd": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                           _i64, _i64, _i64, _i64, _i64, _float, _int, _c_void_p]),
    "pu_attn_bwd_workspace_size": (_size_t, [_i64, _i64, _i64, _i64]),
    "pu_attn_bwd": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                           _c_void_p, _c_void_p, _c_void_p, _c_void_p, _size_t,
                           _i64, _i64, _i64, _i64, _i64, _float, _int, _c_void_p]),
    "pu_attn_bwd_deterministic": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                         _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                         _size_t, _i64, _i64, _i64, _i64, _i64, _float, _int,
                                         _c_void_p]),
    "pu_decode_workspace_size": (_size_t, [_i64, _i64, _i64, _i64]),
    "pu_decode_partial": (_int, [_c_void_p, _int, _c_void_p, _c_void_p, _int, _c_void_p, _i64,
                                 _c_void_p, _c_void_p, _size_t, _i64, _i64, _i64, _i64, _float,
                                 _c_void_p]),
    "pu_decode_combine": (_int, [_c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64,
                                 _c_void_p]),
    "pu_decode": (_int, [_c_void_p, _int, _c_void_p, _c_void_p, _int, _c_void_p, _c_void_p,
                         _c_void_p, _c_void_p, _size_t, _i64, _i64, _i64, _i64, _float,
                         _c_void_p]),
    "pu_decode_noalloc": (_int, [_c_void_p, _int, _c_void_p, _c_void_p, _int, _c_void_p,
                                 _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _float,
                                 _c_void_p]),
    "pu_decode_gqa_workspace_size": (_size_t, [_i64, _i64, _i64, _i64, _i64]),
    "pu_decode_gqa": (_int, [_c_void_p, _int, _c_void_p, _c_void_p, _int, _c_void_p, _c_void_p,
                             _c_void_p, _c_void_p, _size_t, _i64, _i64, _i64, _i64, _i64, _float,
                             _float, _float, _c_void_p]),
    "pu_decode_paged_workspace_size": (_size_t, [_i64, _i64, _i64, _i64, _i64]),
    "pu_decode_paged": (_int, [_c_void_p, _int, _c_void_p, _c_void_p, _int, _c_void_p, _i64,
                               _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _size_t,
                               _i64, _i64, _i64, _float, _c_void_p]),
    "pu_peer_alloc": (_int, [_size_t, ctypes.POINTER(_c_void_p), _c_void_p]),
    "pu_peer_free": (_int, [_c_void_p]),
    "pu_peer_open": (_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "pu_peer_close": (_int, [_c_void_p]),
    "pu_decode_exchange_bytes": (_size_t, [_i64, _i64, _i64, _i64]),
    "pu_decode_push": (_int, [_c_void_p, _int, _c_void_p, _c_void_p, _int, _c_void_p, _i64,
                              _c_void_p, _i64, _i64, ctypes.c_uint32, _c_void_p, _size_t,
                              _i64, _i64, _i64, _i64, _float, _c_void_p]),
    "pu_decode_pull": (_int, [_c_void_p, _i64, ctypes.c_uint32, _c_void_p, _c_void_p, _i64,
                              _i64, _i64, ctypes.c_uint64, _c_void_p]),
    "pu_decode_sharded": (_int, [_c_void_p, _int, _c_void_p, _c_void_p, _int, _c_void_p, _i64,
                                 _c_void_p, _i64, _i64, ctypes.c_uint32, _c_void_p, _c_void_p,
                                 _c_void_p, _size_t, _i64, _i64, _i64, _i64, _float,
                                 ctypes.c_uint64, _c_void_p]),
    "pu_outproj_exchange_bytes": (_size_t, [_i64, _i64, _i64]),
    "pu_outproj_allreduce": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64,
                                    ctypes.c_uint32, _i64, _i64, _i64, ctypes.c_uint64, _c_void_p]),
    "pu_comm_unique_id": (_int, [_c_void_p]),
    "pu_comm_init": (_int, [_c_void_p, _i64, _i64, ctypes.POINTER(_c_void_p)]),
    "pu_allgather_partials": (_int, [_c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p]),
    "pu_comm_destroy": (_int, [_c_void_p]),
    "pu_kv_append": (_int, [_c_void_p, _c_void_p, _int, _c_void_p, _c_void_p, _c_void_p, _i64,
                            _i64, _i64, _c_void_p, _i64, _i64, _i64, _c_void_p]),
}

_lock = threading.Lock()
_lib = None


class PuError(RuntimeError):
    """A nonzero status from libpu_attn (message from pu_last_error)."""

    def __init__(self, code: int, where: str, message: str):
        super().__init__(f"{where} failed with status {code}: {message}")
        self.code = code


def library_path() -> Path:
    return Path(os.environ.get("PU_ATTN_LIB", _LIB_PATH))


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise RuntimeError(
                    f"libpu_attn.so not found at {path}; build it with "
                    "`python pallas-unbound_b200/build.py` (there is no CPU fallback)")
            handle = ctypes.CDLL(str(path))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(code: int, where: str) -> None:
    if code != PU_OK:
        msg = lib().pu_last_error()
        raise PuError(code, where, msg.decode() if msg else "")


def device_status() -> tuple[int, int]:
    """Synchronise the current device and read/clear its kernel status word."""
    detail = _int(0)
    code = lib().pu_device_status(ctypes.byref(detail))
    return code, detail.value
