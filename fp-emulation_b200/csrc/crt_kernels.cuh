// crt_kernels.cuh -- Chinese-remainder reconstruction of the FP64 product
// from its residues, in the reference's floating-point operation order
// (crt_reconstruct.cpp:13-37 / crt_kernel.cu:105-127 of thezettascale/fp-emulation):
// double-double accumulation of r_l * (wh_l + wm_l + wl_l) with TwoProduct and
// TwoSum, q = rint(acc * inv_M), acc - q*M in double-double, then ldexp.
//
// Every operation is an explicit round-to-nearest intrinsic so the compiler
// cannot fuse a multiply into a neighbouring add; the only FMAs are the ones
// the reference writes.  With identical residues this reproduces the
// reference's CPU result bit for bit.
#pragma once

#include "fpemu_device.cuh"

namespace fpemu {

// One accumulation step for residue r (crt_reconstruct.cpp:17-26).
__device__ __forceinline__ void crt_step(double r, double wh, double wm, double wl, double& hi,
                                         double& lo) {
    const double p = __dmul_rn(r, wh);
    const double e = __fma_rn(r, wh, -p);
    const double s = __dadd_rn(hi, p);
    const double v = __dsub_rn(s, hi);
    const double t = __dadd_rn(__dsub_rn(hi, __dsub_rn(s, v)), __dsub_rn(p, v));
    hi = s;
    lo = __dadd_rn(__dadd_rn(__dadd_rn(lo, __fma_rn(r, wm, e)), __dmul_rn(r, wl)), t);
}

// Remove the multiple of M (crt_reconstruct.cpp:29-32); the result is the
// centred integer product in double precision.
__device__ __forceinline__ double crt_finish(double hi, double lo, const CrtConsts& c) {
    const double q = rint(__dmul_rn(__dadd_rn(hi, lo), c.inv_M));
    const double qm = __dmul_rn(q, c.M_hi);
    const double qe = __fma_rn(q, c.M_hi, -qm);
    return __dadd_rn(__dsub_rn(hi, qm), __dsub_rn(__dsub_rn(lo, qe), __dmul_rn(q, c.M_lo)));
}

// Final scaling (crt_reconstruct.cpp:36); a non-finite operand row/column gives NaN.
__device__ __forceinline__ double crt_scale(double x, int re, int ce, int two_bits) {
    if (re == kNonFiniteExp || ce == kNonFiniteExp) return __longlong_as_double(0x7FF8000000000000ll);
    return ldexp(x, re + ce - two_bits);
}

// Standalone reconstruction from uint8 residues [n_mod][m][n] (the debug /
// staged path; the fused GEMM epilogue uses the same three functions).
// Each thread produces 4 consecutive columns of one row.
__global__ void __launch_bounds__(256) crt_kernel(const uint8_t* __restrict__ res, int64_t m,
                                                  int64_t n, int n_mod,
                                                  const int32_t* __restrict__ row_exp,
                                                  const int32_t* __restrict__ col_exp,
                                                  int two_bits, double* __restrict__ C,
                                                  int64_t ldc, const __grid_constant__ CrtConsts cc) {
    const int64_t nq = (n + 3) / 4;
    const int64_t plane = m * n;
    for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < m * nq;
         w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = w / nq;
        const int64_t j0 = (w % nq) * 4;
        const int cnt = (int)min((int64_t)4, n - j0);
        double hi[4] = {0.0, 0.0, 0.0, 0.0}, lo[4] = {0.0, 0.0, 0.0, 0.0};
        const uint8_t* r = res + i * n + j0;
        for (int l = 0; l < n_mod; ++l) {
            const double wh = cc.wh[l], wm = cc.wm[l], wl = cc.wl[l];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (q < cnt) crt_step((double)r[(int64_t)l * plane + q], wh, wm, wl, hi[q], lo[q]);
        }
        const int re = row_exp[i];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (q < cnt)
                C[i * ldc + j0 + q] = crt_scale(crt_finish(hi[q], lo[q], cc), re, col_exp[j0 + q], two_bits);
    }
}

}  // namespace fpemu
