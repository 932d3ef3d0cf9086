"""Ozaki scheme II on INT8 tensor cores -- the drop-in for the reference's
``fp_emulation/ozaki.py`` (thezettascale/fp-emulation), backed by libfpemu.so.

Same public function, same autograd behaviour, same exceptions as
ozaki.py:95-145.  What changed is underneath: one split kernel per operand,
one persistent tcgen05 GEMM whose epilogue reduces every accumulator modulo its
prime and reconstructs FP64 C, all on the caller's current CUDA stream.  CUDA
tensors only: there is no CPU path.

The stage functions (``_split``, ``_matmul_residues``, ``_reconstruct``) keep
the reference's step boundaries so each step can be compared with the
reference on its own; the production call goes through one C entry point.
"""
from __future__ import annotations

import ctypes
import os

import torch

from fp_emulation import _lib

# ozaki.py:6-9
_PRIMES = [
    3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53,
    59, 61, 67, 71, 73, 79, 83, 89, 97, 101, 103, 107, 109, 113, 127,
]

# ozaki.py:12-17
_PRECISION_BITS = {
    torch.float16: 11,
    torch.bfloat16: 8,
    torch.float32: 24,
    torch.float64: 53,
}

# How device-side failures (a bounded wait in a kernel that ran out) surface.
# Such a failure also writes NaN over the output tiles the kernel could not finish.
#   default ("poll"): every call ends by looking, without synchronising, at the
#       host copy of the device's error record and raises FpemuError if a kernel
#       that has already finished recorded one -- like an asynchronous CUDA
#       error, a failure surfaces in the first call that ends after it happened;
#   FPEMU_CHECK=1: also synchronise after every call and raise at once;
#   FPEMU_CHECK=0: no check (the caller reads fp_emulation._lib.device_error()).
_CHECK_MODE = {"0": "off", "1": "sync"}.get(os.environ.get("FPEMU_CHECK", ""), "poll")


def _n_moduli(k, bits):
    """ozaki.py:20-29 through fpemu_plan_moduli; ValueError when the primes run out."""
    n = ctypes.c_int(0)
    _lib.check(_lib.load().fpemu_plan_moduli(int(k), int(bits), ctypes.byref(n), None), "_n_moduli")
    return n.value


def _crt_weights(moduli):
    """ozaki.py:62-80 through fpemu_crt_weights (exact 128-bit integer arithmetic).
    ``moduli`` must be a prefix of ``_PRIMES``, as the reference always uses."""
    n = len(moduli)
    if list(moduli) != _PRIMES[:n]:
        raise ValueError("moduli must be the leading primes 3, 5, 7, ...")
    arrs = [(ctypes.c_double * n)() for _ in range(3)]
    scal = [ctypes.c_double() for _ in range(3)]
    _lib.check(_lib.load().fpemu_crt_weights(n, *arrs, *[ctypes.byref(s) for s in scal]), "_crt_weights")
    return list(arrs[0]), list(arrs[1]), list(arrs[2]), scal[0].value, scal[1].value, scal[2].value


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*tensors):
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                "fp_emulation (B200 build) runs on CUDA tensors only; got a tensor on "
                f"{t.device}. Move the operands to a CUDA device.")
    dev = tensors[0].device
    for t in tensors[1:]:
        if t.device != dev:
            raise RuntimeError(f"operands on different devices: {dev} and {t.device}")
    if _CHECK_MODE != "off" and dev.index not in _lib._watched:
        with torch.cuda.device(dev):
            _lib.watch(dev.index)
    return dev


def _res_ld(k: int) -> int:
    return ((k + 15) // 16) * 16


def _after_call(what: str, dev) -> None:
    """Surface a device-side failure recorded on `dev` (see _CHECK_MODE)."""
    if _CHECK_MODE == "off":
        return
    with torch.cuda.device(dev):
        if _CHECK_MODE == "poll" and _lib.poll_error()[0] == 0:
            return
        code, where, block, detail = _lib.device_error(clear=True)
    if code:
        raise _lib.FpemuError(code, f"{what}: a kernel of fp_emulation on {dev} gave up waiting (where={where} "
                                    f"block={block} detail={detail}); the outputs it could not finish are NaN")


# ------------------------------------------------------------------ stages --

def _split(X, bits, n_mod):
    """ozaki.py:32-46 for one operand, fused on the GPU: returns
    (residues int8 [n_mod, rows, res_ld] with K contiguous, exps int32 [rows]).

    ``X`` is [rows, k]; for the reference's B [k, n] pass ``B.T``.  Residues
    equal ``(round(ldexp(X, bits - exp)) mod p)`` in [0, p); the columns past k
    are zero.
    """
    dev = _require_cuda(X)
    X = X.double()
    rows, k = X.shape
    ld = _res_ld(k)
    res = torch.empty((n_mod, rows, ld), dtype=torch.int8, device=dev)
    exps = torch.empty((rows,), dtype=torch.int32, device=dev)
    colmax = torch.empty((max(rows, 1),), dtype=torch.int64, device=dev) if X.stride(1) != 1 else None
    with torch.cuda.device(dev):
        st = _lib.load().fpemu_split(rows, k, X.data_ptr(), X.stride(0), X.stride(1), bits, n_mod,
                                     res.data_ptr(), ld, rows * ld, exps.data_ptr(),
                                     None if colmax is None else colmax.data_ptr(), _stream(dev))
    _lib.check(st, "_split")
    _after_call("_split", dev)
    return res, exps


def _scale_to_int_residues(A, B, bits, n_mod):
    """The reference's _scale_to_int + _residues for both operands (ozaki.py:111-113)."""
    a_res, row_exp = _split(A, bits, n_mod)
    b_res, col_exp = _split(B.T, bits, n_mod)
    return a_res, b_res, row_exp, col_exp


def _matmul_residues(a_res, b_res, moduli, raw=False):
    """ozaki.py:49-59: per-modulus products of the K-major residue planes.
    ``raw=False`` gives (a_l @ b_l^T) mod p_l as uint8 [n_mod, m, n] (the
    reference returns the same values as int32); ``raw=True`` gives the int32
    products before the reduction."""
    dev = _require_cuda(a_res, b_res)
    n_mod, m, ld = a_res.shape
    n = b_res.shape[1]
    k = ld  # zero columns past the true k contribute nothing
    out = torch.empty((n_mod, m, n), dtype=torch.int32 if raw else torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = _lib.load().fpemu_gemm_residues(m, n, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), ld,
                                             0 if raw else 1, out.data_ptr(), None, 0, _stream(dev))
    _lib.check(st, "_matmul_residues")
    _after_call("_matmul_residues", dev)
    return out


def _reconstruct(residues, moduli, bits, row_exp, col_exp):
    """ozaki.py:83-92: CRT reconstruction from uint8 residues [n_mod, m, n]."""
    dev = _require_cuda(residues, row_exp, col_exp)
    res = residues.to(torch.uint8).contiguous()
    n_mod, m, n = res.shape
    out = torch.empty((m, n), dtype=torch.float64, device=dev)
    re = row_exp.to(torch.int32).contiguous()
    ce = col_exp.to(torch.int32).contiguous()
    with torch.cuda.device(dev):
        st = _lib.load().fpemu_crt_reconstruct(m, n, n_mod, res.data_ptr(), re.data_ptr(), ce.data_ptr(),
                                               bits, out.data_ptr(), n, _stream(dev))
    _lib.check(st, "_reconstruct")
    _after_call("_reconstruct", dev)
    return out


# --------------------------------------------------------------- forward ----

def _workspace(m, n, k, n_mod, dev):
    nbytes = _lib.load().fpemu_workspace_size(m, n, k, n_mod)
    if nbytes == 0:
        raise _lib.FpemuError(_lib.FPEMU_ERR_NO_DEVICE, "fpemu_workspace_size failed: "
                              + _lib.load().fpemu_last_error().decode(errors="replace"))
    return torch.empty((nbytes,), dtype=torch.uint8, device=dev)


def _fused_output(orig_dtype, bias, n, dev):
    """(c_dtype, torch dtype of C, bias to pass) for the fused epilogue: float64
    and float32 outputs are written by the kernel (the float32 one rounded from
    the double result, as ``.to(torch.float32)`` does), with the bias added in
    the output's type; other dtypes come back as float64 for torch to finish."""
    if orig_dtype == torch.float32:
        c_dtype, out_dtype = _lib.FPEMU_C_F32, torch.float32
    else:
        c_dtype, out_dtype = _lib.FPEMU_C_F64, torch.float64
    fused_bias = None
    if bias is not None and orig_dtype in (torch.float32, torch.float64):
        if bias.shape != (n,):
            raise RuntimeError(f"bias of shape {tuple(bias.shape)} does not match {n} output columns")
        fused_bias = bias.to(device=dev, dtype=out_dtype).contiguous()
    return c_dtype, out_dtype, fused_bias


def _dtype_bits(dtype):
    """ozaki.py:97-104: the precision bits of a float dtype, TypeError otherwise."""
    bits = _PRECISION_BITS.get(dtype)
    if bits is None:
        supported = ", ".join(str(d) for d in _PRECISION_BITS)
        raise TypeError(
            f"unsupported dtype {dtype}. "
            f"CRT matmul emulates floating-point precision via int8 arithmetic; "
            f"input must be a float type ({supported})"
        )
    return bits


def _ozaki2_forward(A, B, n_mod=None, bias=None):
    """ozaki.py:95-119: scale -> modular INT8 matmuls -> CRT reconstruct, as one
    C call (split A, split B, fused GEMM + CRT) on the current stream.
    ``n_mod`` overrides the reference's modulus count (for sweeps).  ``bias``
    (n values) is added after the cast to the input's dtype -- nn.py:20-21's
    ``out + self.bias`` -- fused into the epilogue for float64/float32."""
    bits = _dtype_bits(A.dtype)
    dev = _require_cuda(A, B)
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[0]:
        raise RuntimeError(f"ozaki2_int8_matmul: expected [m,k] @ [k,n], got {tuple(A.shape)} @ {tuple(B.shape)}")
    orig_dtype = A.dtype
    A, B = A.double(), B.double()
    m, k = A.shape
    n = B.shape[1]
    if k == 0:
        raise RuntimeError("ozaki2_int8_matmul: inner dimension k must be non-zero "
                           "(the reference's amax over an empty dimension fails the same way)")
    if n_mod is None:
        n_mod = _n_moduli(k, bits)
    c_dtype, out_dtype, fused_bias = _fused_output(orig_dtype, bias, n, dev)
    C = torch.empty((m, n), dtype=out_dtype, device=dev)
    if m and n:
        with torch.cuda.device(dev):
            ws = _workspace(m, n, k, n_mod, dev)
            st = _lib.load().fpemu_ozaki2_gemm_ex(
                m, n, k, A.data_ptr(), A.stride(0), A.stride(1), B.data_ptr(), B.stride(0), B.stride(1),
                C.data_ptr(), n, c_dtype, None if fused_bias is None else fused_bias.data_ptr(), bits, n_mod,
                ws.data_ptr(), ws.numel(), _stream(dev))
        _lib.check(st, "ozaki2_int8_matmul")
        _after_call("ozaki2_int8_matmul", dev)
    elif fused_bias is not None:
        C += fused_bias
    if C.dtype != orig_dtype:
        C = C.to(orig_dtype)
    if bias is not None and fused_bias is None:
        C = C + bias
    return C


class PreparedOperand:
    """A static operand of ozaki2_int8_matmul whose split is kept on the GPU.

    ``prepare_operand(X, "left")`` for the A of ``A @ B`` ([m, k]), or
    ``prepare_operand(X, "right")`` for the B ([k, n]).  The first product that
    uses it splits X (scaling exponents and int8 residues, ozaki.py:32-46) and
    keeps the split -- n_mod bytes per element plus one int32 per row or column
    -- so later products split only the other operand: the Chebyshev
    differentiation matrix D of ``D @ u`` applied to new fields every epoch, or
    the weight of a Linear layer.  The split is redone when X's storage or
    version changes (an in-place update, an optimizer step) or the product needs
    another modulus count or precision.  Results are bit-identical to the
    unprepared product.  Under autograd the backward products use ``.T``, the
    transposed operand, itself prepared on first use.  Not in the reference,
    which splits both operands on every call."""

    def __init__(self, X, side):
        if side not in ("left", "right"):
            raise ValueError(f"side must be 'left' or 'right', got {side!r}")
        if not isinstance(X, torch.Tensor) or X.dim() != 2:
            raise RuntimeError("a prepared operand is a 2-D tensor")
        _dtype_bits(X.dtype)
        _require_cuda(X)
        self.tensor = X
        self.side = side
        self._split = None  # (key, residues, exponents)
        self._t = None

    @property
    def shape(self):
        return self.tensor.shape

    @property
    def dtype(self):
        return self.tensor.dtype

    @property
    def device(self):
        return self.tensor.device

    @property
    def T(self):
        """The transposed operand, prepared for the same side (cached): the
        backward of ``A @ B`` computes ``A.T @ grad`` and ``grad @ B.T``."""
        if self._t is None:
            self._t = PreparedOperand(self.tensor.T, self.side)
            self._t._t = self
        return self._t

    def residues(self, n_mod, bits):
        """(int8 residues [n_mod, rows, ld], int32 exponents [rows]) of the rows
        of X (left) or the columns of X (right), split once per version."""
        X = self.tensor
        key = (X.data_ptr(), X._version, tuple(X.stride()), X.device, n_mod, bits)
        if self._split is None or self._split[0] != key:
            Xd = X.detach().double()
            res, exps = _split(Xd if self.side == "left" else Xd.T, bits, n_mod)
            self._split = (key, res, exps)
        return self._split[1], self._split[2]


def prepare_operand(X, side="left"):
    """Keep the split of the static operand X on the GPU for repeated products
    (see PreparedOperand)."""
    return PreparedOperand(X, side)


def _ozaki2_forward_prepared(A, B, bias=None):
    """_ozaki2_forward where A and/or B is a PreparedOperand: the prepared side's
    cached split, the other side split here, then the fused GEMM + CRT.  Same
    dtype rules, output and bias handling as _ozaki2_forward."""
    pa, pb = isinstance(A, PreparedOperand), isinstance(B, PreparedOperand)
    if pa and A.side != "left":
        raise ValueError("the left operand was prepared as a right operand")
    if pb and B.side != "right":
        raise ValueError("the right operand was prepared as a left operand")
    At = A.tensor if pa else A
    Bt = B.tensor if pb else B
    bits = _dtype_bits(At.dtype)
    dev = _require_cuda(At, Bt)
    if At.dim() != 2 or Bt.dim() != 2 or At.shape[1] != Bt.shape[0]:
        raise RuntimeError(f"ozaki2_int8_matmul: expected [m,k] @ [k,n], got {tuple(At.shape)} @ {tuple(Bt.shape)}")
    orig_dtype = At.dtype
    m, k = At.shape
    n = Bt.shape[1]
    if k == 0:
        raise RuntimeError("ozaki2_int8_matmul: inner dimension k must be non-zero")
    n_mod = _n_moduli(k, bits)
    c_dtype, out_dtype, fused_bias = _fused_output(orig_dtype, bias, n, dev)
    C = torch.empty((m, n), dtype=out_dtype, device=dev)
    if m and n:
        a_res, row_exp = A.residues(n_mod, bits) if pa else _split(At.double(), bits, n_mod)
        b_res, col_exp = B.residues(n_mod, bits) if pb else _split(Bt.double().T, bits, n_mod)
        ld = a_res.shape[2]
        lib = _lib.load()
        with torch.cuda.device(dev):
            ws = torch.empty((max(lib.fpemu_gemm_workspace_size(m, n, n_mod), 256),), dtype=torch.uint8, device=dev)
            st = lib.fpemu_gemm_crt_ex(m, n, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), ld, b_res.stride(0),
                                       row_exp.data_ptr(), col_exp.data_ptr(), bits, C.data_ptr(), n, c_dtype,
                                       None if fused_bias is None else fused_bias.data_ptr(), 0, ws.data_ptr(),
                                       ws.numel(), _stream(dev))
        _lib.check(st, "ozaki2_int8_matmul (prepared operand)")
        _after_call("ozaki2_int8_matmul", dev)
    elif fused_bias is not None:
        C += fused_bias
    if C.dtype != orig_dtype:
        C = C.to(orig_dtype)
    if bias is not None and fused_bias is None:
        C = C + bias
    return C


class _OzakiMatmul(torch.autograd.Function):
    """ozaki.py:122-136: backward re-enters the emulated product twice."""

    @staticmethod
    def forward(A, B):
        return _ozaki2_forward(A, B)

    @staticmethod
    def setup_context(ctx, inputs, output):
        ctx.save_for_backward(*inputs)

    @staticmethod
    def backward(ctx, grad):
        A, B = ctx.saved_tensors
        grad_A = ozaki2_int8_matmul(grad, B.T) if ctx.needs_input_grad[0] else None
        grad_B = ozaki2_int8_matmul(A.T, grad) if ctx.needs_input_grad[1] else None
        return grad_A, grad_B


class _OzakiMatmulPrepared(torch.autograd.Function):
    """_OzakiMatmul with one or both operands prepared; the backward products use
    the prepared transposes (ozaki.py:132-136 otherwise)."""

    @staticmethod
    def forward(A_t, B_t, A_op, B_op):
        return _ozaki2_forward_prepared(A_op, B_op)

    @staticmethod
    def setup_context(ctx, inputs, output):
        A_t, B_t, A_op, B_op = inputs
        ctx.save_for_backward(A_t, B_t)
        ctx.ops = (A_op, B_op)

    @staticmethod
    def backward(ctx, grad):
        A_t, B_t = ctx.saved_tensors
        A_op, B_op = ctx.ops
        B_T = B_op.T if isinstance(B_op, PreparedOperand) else B_t.T
        A_T = A_op.T if isinstance(A_op, PreparedOperand) else A_t.T
        grad_A = ozaki2_int8_matmul(grad, B_T) if ctx.needs_input_grad[0] else None
        grad_B = ozaki2_int8_matmul(A_T, grad) if ctx.needs_input_grad[1] else None
        return grad_A, grad_B, None, None


def ozaki2_int8_matmul(A, B):
    """
    FP-accurate matmul via INT8 tensor cores (Ozaki scheme II + CRT).

    Precision matches input dtype (fp16, bf16, fp32, fp64).  CUDA tensors only.
    Either operand may be a PreparedOperand (prepare_operand), whose split is
    reused across calls.
    """
    if isinstance(A, PreparedOperand) or isinstance(B, PreparedOperand):
        A_t = A.tensor if isinstance(A, PreparedOperand) else A
        B_t = B.tensor if isinstance(B, PreparedOperand) else B
        return _OzakiMatmulPrepared.apply(A_t, B_t, A, B)
    return _OzakiMatmul.apply(A, B)
