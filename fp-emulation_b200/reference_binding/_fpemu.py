"""ctypes binding of libfpemu.so for the reference package (thezettascale/fp-emulation).

This is the file a maintainer of the reference would add as
``src/fp_emulation/_fpemu.py``; it replaces the CUDA branch of
``_ozaki2_forward`` (ozaki.py:95-119, which today calls ``_cuda_crt.py``'s
cuBLASLt batched GEMM and CRT kernel) with one C call into libfpemu.so.  The
reference's CPU branch is unchanged.  The library path comes from FPEMU_LIB.

In ``ozaki.py:_ozaki2_forward``, right after ``moduli = _PRIMES[:n_mod]``
(ozaki.py:109), the reference adds::

    if A.is_cuda:
        from fp_emulation._fpemu import cuda_ozaki2
        result = cuda_ozaki2(A, B, bits, n_mod)
        return result if orig_dtype == torch.float64 else result.to(orig_dtype)
"""
import ctypes
import os

import torch

_lib = ctypes.CDLL(os.environ.get("FPEMU_LIB", "libfpemu.so"))
_i64, _int, _sz, _vp = ctypes.c_int64, ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p
_lib.fpemu_workspace_size.restype = _sz
_lib.fpemu_workspace_size.argtypes = [_i64, _i64, _i64, _int]
_lib.fpemu_ozaki2_dgemm.restype = _int
_lib.fpemu_ozaki2_dgemm.argtypes = [_i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64,
                                    _vp, _i64, _int, _int, _vp, _sz, _vp]
_lib.fpemu_last_error.restype = ctypes.c_char_p


def cuda_ozaki2(A, B, bits, n_mod):
    """A [m,k] @ B [k,n], float64 CUDA tensors of any strides -> float64 [m,n]."""
    m, k = A.shape
    n = B.shape[1]
    C = torch.empty((m, n), dtype=torch.float64, device=A.device)
    if m == 0 or n == 0:
        return C
    with torch.cuda.device(A.device):
        ws = torch.empty(_lib.fpemu_workspace_size(m, n, k, n_mod), dtype=torch.uint8, device=A.device)
        st = _lib.fpemu_ozaki2_dgemm(m, n, k, A.data_ptr(), A.stride(0), A.stride(1),
                                     B.data_ptr(), B.stride(0), B.stride(1), C.data_ptr(), n,
                                     bits, n_mod, ws.data_ptr(), ws.numel(),
                                     torch.cuda.current_stream(A.device).cuda_stream)
    if st != 0:
        raise RuntimeError(_lib.fpemu_last_error().decode())
    return C
