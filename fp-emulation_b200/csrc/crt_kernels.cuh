// crt_kernels.cuh -- Chinese-remainder reconstruction of the FP64 product
// from its residues, in the reference's floating-point operation order
// (crt_reconstruct.cpp:13-37 / crt_kernel.cu:105-127 of thezettascale/fp-emulation):
// double-double accumulation of r_l * (wh_l + wm_l + wl_l) with TwoProduct and
// an exact two-sum, q = rint(acc * inv_M), acc - q*M in double-double, then ldexp.
//
// Every operation is an explicit round-to-nearest intrinsic so the compiler
// cannot fuse a multiply into a neighbouring add; the only FMAs are the ones
// the reference writes.  With identical residues this reproduces the
// reference's CPU result bit for bit.
#pragma once

#include "fpemu_device.cuh"

namespace fpemu {

// One accumulation step for residue r (crt_reconstruct.cpp:17-26).
//
// The reference takes the rounding error t of s = hi + p with TwoSum (six
// operations).  Here both addends are non-negative -- residues and CRT weights
// are, so every p and every partial sum hi is -- hence their order by magnitude
// is the order of their bit patterns, picked with integer compares, and Fast2Sum
// on (larger, smaller) gives the same exact error in two operations (Dekker:
// for |a| >= |b|, s - a and b - (s - a) are exact).  Both forms yield the exact
// value of (hi + p) - s, a representable double, so t and everything after it
// are bit-identical to the reference's.
__device__ __forceinline__ void crt_step(double r, double wh, double wm, double wl, double& hi,
                                         double& lo) {
    const double p = __dmul_rn(r, wh);
    const double e = __fma_rn(r, wh, -p);
    const double s = __dadd_rn(hi, p);
    const unsigned long long hb = (unsigned long long)__double_as_longlong(hi);
    const unsigned long long pb = (unsigned long long)__double_as_longlong(p);
    const double big = __longlong_as_double((long long)(hb > pb ? hb : pb));
    const double small = __longlong_as_double((long long)(hb > pb ? pb : hb));
    const double t = __dsub_rn(small, __dsub_rn(s, big));
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

// Standalone reconstruction from uint8 residues [n_mod][m][n] (the parity tap
// of the reference's _reconstruct, and the second kernel of the split path).
// A thread produces 16 consecutive columns of one row: 16-byte residue loads
// per modulus when n is a multiple of 16, byte loads otherwise.  Output as in
// the fused epilogue: double, or its float rounding, then the optional bias in
// C's type, columns optionally scattered in segments (see GemmParams).  An
// output with a residue byte >= 128 -- never a residue (p <= 127); the residue
// GEMM writes 0xFF over units it could not finish -- becomes NaN.
__global__ void __launch_bounds__(256) crt_kernel(const __grid_constant__ CrtParams P) {
    const int64_t nq = (P.n + 15) / 16;
    const int64_t plane = P.m * P.n;
    const bool vec = (P.n % 16) == 0 && (reinterpret_cast<uintptr_t>(P.res) % 16) == 0;
    for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < P.m * nq;
         w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = w / nq;
        const int64_t j0 = (w - i * nq) * 16;
        const int cnt = (int)min((int64_t)16, P.n - j0);
        double hi[16], lo[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) { hi[q] = 0.0; lo[q] = 0.0; }
        uint32_t seen[4] = {0u, 0u, 0u, 0u};  // OR of every modulus's bytes: bit 7 marks a non-residue
        const uint8_t* r = P.res + i * P.n + j0;
#pragma unroll 1
        for (int l = 0; l < P.n_mod; ++l) {
            const double wh = P.cc.wh[l], wm = P.cc.wm[l], wl = P.cc.wl[l];
            uint32_t b[4];
            if (vec) {
                const uint4 v = __ldcs(reinterpret_cast<const uint4*>(r + (int64_t)l * plane));
                b[0] = v.x; b[1] = v.y; b[2] = v.z; b[3] = v.w;
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t x = 0;
                    for (int e = 0; e < 4; ++e)
                        if (4 * q + e < cnt) x |= (uint32_t)r[(int64_t)l * plane + 4 * q + e] << (8 * e);
                    b[q] = x;
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) seen[q] |= b[q];
#pragma unroll
            for (int q = 0; q < 16; ++q)
                crt_step((double)((b[q >> 2] >> (8 * (q & 3))) & 0xFFu), wh, wm, wl, hi[q], lo[q]);
        }
        const int re = P.row_exp[i];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            if (q < cnt) {
                const int64_t j = j0 + q;
                double v = crt_scale(crt_finish(hi[q], lo[q], P.cc), re, P.col_exp[j], P.two_bits);
                if ((seen[q >> 2] >> (8 * (q & 3))) & 0x80u) v = __longlong_as_double(0x7FF8000000000000ll);
                const int64_t oc = P.col_seg > 0 ? (j / P.col_seg) * P.col_seg_stride + j % P.col_seg : j;
                if (P.c_f32) {
                    float f = __double2float_rn(v);
                    if (P.bias) f = __fadd_rn(f, static_cast<const float*>(P.bias)[j]);
                    static_cast<float*>(P.C)[i * P.ldc + oc] = f;
                } else {
                    if (P.bias) v = __dadd_rn(v, static_cast<const double*>(P.bias)[j]);
                    static_cast<double*>(P.C)[i * P.ldc + oc] = v;
                }
            }
        }
    }
}

}  // namespace fpemu
