"""fp_emulation -- B200 (sm_100a) build of Ozaki scheme II FP64 emulation.

Drop-in for the reference package's GEMM path (its ``__init__.py:1-13``):
``ozaki2_int8_matmul``, ``Linear`` and ``convert``.  The reference's ML-PLAC
helpers (fit_pwl, eval_pwl, ...) are not part of this build.
"""
from fp_emulation.nn import Linear, convert
from fp_emulation.ozaki import PreparedOperand, ozaki2_int8_matmul, prepare_operand

__all__ = ["Linear", "convert", "ozaki2_int8_matmul", "PreparedOperand", "prepare_operand"]
