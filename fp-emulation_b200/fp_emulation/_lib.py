"""ctypes binding of libfpemu.so, the C ABI declared in include/fpemu.h.

This is the only way the Python layer reaches the GPU: plain pointers, sizes,
strides and a CUDA stream handle.  The library is built in-tree by
``fp-emulation_b200/build.py``; if it is missing, loading fails loudly (there
is no CPU fallback).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libfpemu.so")
ABI_VERSION = 1

FPEMU_OK = 0
FPEMU_ERR_INVALID = 1
FPEMU_ERR_NO_MODULI = 2
FPEMU_ERR_UNSUPPORTED = 3
FPEMU_ERR_WORKSPACE = 4
FPEMU_ERR_CUDA = 5
FPEMU_ERR_TIMEOUT = 6
FPEMU_ERR_NO_DEVICE = 7
FPEMU_C_F64 = 0
FPEMU_C_F32 = 1

# Every symbol include/fpemu.h declares, with its ctypes signature.
_i64, _int, _sz, _vp, _dp = ctypes.c_int64, ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_double
_IP = ctypes.POINTER(ctypes.c_int)
SIGNATURES = {
    "fpemu_status_string": (ctypes.c_char_p, [_int]),
    "fpemu_last_error": (ctypes.c_char_p, []),
    "fpemu_abi_version": (_int, []),
    "fpemu_plan_moduli": (_int, [_i64, _int, _IP, _vp]),
    "fpemu_crt_weights": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _vp]),
    "fpemu_max_k": (_i64, [_int]),
    "fpemu_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "fpemu_ozaki2_dgemm": (_int, [_i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
                                  _int, _int, _vp, _sz, _vp]),
    "fpemu_split": (_int, [_i64, _i64, _vp, _i64, _i64, _int, _int, _vp, _i64, _i64, _vp, _vp, _vp]),
    "fpemu_gemm_residues": (_int, [_i64, _i64, _i64, _int, _vp, _vp, _i64, _int, _vp, _vp, _sz, _vp]),
    "fpemu_crt_reconstruct": (_int, [_i64, _i64, _int, _vp, _vp, _vp, _int, _vp, _i64, _vp]),
    "fpemu_gemm_crt": (_int, [_i64, _i64, _i64, _int, _vp, _vp, _i64, _i64, _vp, _vp, _int, _vp, _i64,
                              _int, _vp, _sz, _vp]),
    "fpemu_gemm_workspace_size": (_sz, [_i64, _i64, _int]),
    "fpemu_gemm_kernels": (_int, [_i64, _i64]),
    "fpemu_ozaki2_gemm_ex": (_int, [_i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _int, _vp,
                                    _int, _int, _vp, _sz, _vp]),
    "fpemu_gemm_crt_ex": (_int, [_i64, _i64, _i64, _int, _vp, _vp, _i64, _i64, _vp, _vp, _int, _vp, _i64,
                                 _int, _vp, _int, _vp, _sz, _vp]),
    "fpemu_gemm_crt_segmented": (_int, [_i64, _i64, _i64, _int, _vp, _vp, _i64, _i64, _vp, _vp, _int, _vp, _i64,
                                        _i64, _i64, _int, _vp, _sz, _vp]),
    "fpemu_gemm_crt_noalloc": (_int, [_i64, _i64, _i64, _int, _vp, _vp, _i64, _vp, _vp, _int, _vp, _i64, _vp]),
    "fpemu_device_error": (_int, [_IP, _IP, _IP, _IP, _int]),
    "fpemu_watch_errors": (_int, []),
    "fpemu_poll_error": (_int, [_IP, _IP, _IP, _IP]),
}

_lock = threading.RLock()
_lib = None


class FpemuError(RuntimeError):
    """A failed libfpemu call (CUDA error, device timeout, bad workspace...)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def load():
    """Load libfpemu.so once and attach the ctypes signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python fp-emulation_b200/build.py` "
                    "(fp_emulation has no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.fpemu_abi_version() != ABI_VERSION:
                raise ImportError(f"libfpemu ABI {lib.fpemu_abi_version()} != {ABI_VERSION}")
            _lib = lib
    return _lib


def check(status: int, what: str = "") -> None:
    """Raise the exception the reference would raise for this status."""
    if status == FPEMU_OK:
        return
    lib = load()
    msg = lib.fpemu_last_error().decode(errors="replace") or lib.fpemu_status_string(status).decode()
    if what:
        msg = f"{what}: {msg}"
    if status == FPEMU_ERR_NO_MODULI:
        raise ValueError(msg)  # ozaki.py:29
    if status == FPEMU_ERR_INVALID:
        raise ValueError(msg)
    raise FpemuError(status, msg)


def device_error(clear: bool = True):
    """(code, where, block, detail) of the first device-side failure (0 = none).
    Synchronises the current device."""
    lib = load()
    vals = [ctypes.c_int(0) for _ in range(4)]
    check(lib.fpemu_device_error(*[ctypes.byref(v) for v in vals], int(clear)), "device_error")
    return tuple(v.value for v in vals)


_watched = set()


def watch(device_index: int) -> None:
    """Once per device (which must be current): have this library's kernels also
    record their first failure in pinned host memory, readable by poll_error()
    without synchronising."""
    if device_index in _watched:
        return
    lib = load()
    with _lock:
        if device_index not in _watched:
            check(lib.fpemu_watch_errors(), "fpemu_watch_errors")
            _watched.add(device_index)


def poll_error():
    """(code, where, block, detail) of the first failure recorded on the current
    device by kernels that have already finished; does not synchronise.  Needs
    watch() on this device."""
    lib = load()
    vals = [ctypes.c_int(0) for _ in range(4)]
    check(lib.fpemu_poll_error(*[ctypes.byref(v) for v in vals]), "poll_error")
    return tuple(v.value for v in vals)
