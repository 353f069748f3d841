"""Loads ``libgdn_b200.so`` (the sm_100a kernels behind the C ABI of
``include/gdn_b200.h``) with ctypes and declares its entry points.

There is no fallback: if the library is missing or cannot be loaded, every
call raises, so a run never silently takes another path.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgdn_b200.so")

GDN_OK = 0
GDN_ERR_INVALID = 1
GDN_ERR_UNSUPPORTED = 2
GDN_ERR_ALIGN = 3
GDN_ERR_CUDA = 4
GDN_ERR_DEVICE = 5
GDN_ERR_TOO_LARGE = 6

_vp, _f, _i = ctypes.c_void_p, ctypes.c_float, ctypes.c_int

# (name, restype, argtypes) for every function declared in include/*.h
SIGNATURES = {
    "gdn_abi_version": (_i, []),
    "gdn_strerror": (ctypes.c_char_p, [_i]),
    "gdn_device_status": (_i, [_i]),
    "gdn_decode_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f,
                            _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "gdn_decode_fwd_host": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f,
                                 _i, _i, _i, _i, _i, _vp, _vp, _vp, ctypes.c_size_t, _i, _vp]),
    "gdn_decode_host_workspace_bytes": (ctypes.c_size_t, [_i, _i, _i]),
    "gdn_prefill_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                             _i, _i, _f, _i, _i, _i, _i, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "gdn_prefill_fwd_checkpointed": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                                          _i, _i, _f, _i, _i, _i, _i, _vp, _vp,
                                          _vp, _vp, ctypes.c_longlong, _i, _vp, ctypes.c_size_t, _vp]),
    "gdn_prefill_fwd_ex": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                                _i, _i, _f, _i, _i, _i, _i, _vp, _vp,
                                _vp, _vp, ctypes.c_longlong, _i, _i, _vp, ctypes.c_size_t, _vp]),
    "gdn_prefill_fwd_host": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                                  _i, _i, _f, _i, _i, _i, _i, _vp, _vp, _vp, ctypes.c_size_t, _i, _vp]),
    "gdn_prefill_host_workspace_bytes": (ctypes.c_size_t, [_i, _i, _i, _i, _i]),
    "gdn_prefill_workspace_bytes": (ctypes.c_size_t, [_i, _i, _i, _i]),
    "gdn_prefill_fwd_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i,
                                     _i, _i, _f, _i, _i, _i, _i, _vp, _vp, _vp]),
    "gdn_mtp_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _vp, _vp, _vp, _vp, _f,
                         _i, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _vp]),
    "gdn_umma_selftest": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "gdn_umma_selftest_ex": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, ctypes.c_longlong, _vp]),
}

_lib = None


class GDNError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed with status {status}: {strerror(status)}")


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with "
                "`python -m rocm_flashinfer_contest_b200.build` (needs nvcc)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def strerror(status: int) -> str:
    return lib().gdn_strerror(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != GDN_OK:
        raise GDNError(fn, status)
