/*
 * crt_oracle.c -- CPU restatement of the reference's CRT reconstruction.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path; it is never linked into, loaded by, or called from the product
 * library.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg load it.
 *
 * It restates fp_emulation/csrc/crt_reconstruct.cpp:6-38 of the reference
 * (thezettascale/fp-emulation).  The floating-point operation sequence has to
 * be the same one, in the same order, because the point of this oracle is a
 * bit-exact comparison: per element, a double-double accumulation of
 * r_k * (wh_k + wm_k + wl_k) using TwoProduct (one fma) and TwoSum, then the
 * quotient q = rint(acc * inv_M), the subtraction of q*M in double-double,
 * and a final ldexp by row_exp[i] + col_exp[j] - two_bits.
 *
 * Build with -ffp-contract=off: the reference builds through
 * torch.utils.cpp_extension with -std=c++17, where GCC does not contract
 * a*b+c, so the only fused multiply-adds are the explicit fma() calls.
 */
#include <math.h>
#include <stdint.h>

/*
 * Per-element body, crt_reconstruct.cpp:14-36.  Residues come either as int32
 * (the reference's layout) or as uint8 (the layout the CUDA path stages);
 * exactly one of r32 / r8 is non-NULL.
 */
static inline double crt_one(const int32_t *r32, const uint8_t *r8, int64_t plane, int64_t idx,
                             const double *wh, const double *wm, const double *wl,
                             double M_hi, double M_lo, double inv_M, int n_mod) {
    double hi = 0.0, lo = 0.0;
    for (int k = 0; k < n_mod; ++k) {
        const int64_t at = (int64_t)k * plane + idx;
        const double r = r32 ? (double)r32[at] : (double)r8[at];
        const double p = r * wh[k];            /* TwoProduct: p + e == r*wh exactly */
        const double e = fma(r, wh[k], -p);
        const double s = hi + p;               /* TwoSum(hi, p) -> s + t */
        const double v = s - hi;
        const double t = (hi - (s - v)) + (p - v);
        hi = s;
        lo = lo + fma(r, wm[k], e) + r * wl[k] + t;
    }
    const double q = rint((hi + lo) * inv_M);
    const double qm = q * M_hi;
    const double qe = fma(q, M_hi, -qm);
    return (hi - qm) + (lo - qe - q * M_lo);
}

static void crt_all(const int32_t *r32, const uint8_t *r8, const double *wh, const double *wm,
                    const double *wl, double M_hi, double M_lo, double inv_M,
                    const int32_t *row_exp, const int32_t *col_exp, int two_bits, double *out,
                    int64_t rows, int64_t cols, int n_mod) {
    const int64_t n = rows * cols;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < n; ++idx) {
        const int64_t i = idx / cols, j = idx % cols;
        const double x = crt_one(r32, r8, n, idx, wh, wm, wl, M_hi, M_lo, inv_M, n_mod);
        out[idx] = ldexp(x, row_exp[i] + col_exp[j] - two_bits);
    }
}

/*
 * residues: [n_mod][rows][cols] (plane stride rows*cols), values in [0, p_k).
 * out: float64 [rows][cols].
 */
void oracle_crt_reconstruct(const int32_t *residues, const double *wh, const double *wm,
                            const double *wl, double M_hi, double M_lo, double inv_M,
                            const int32_t *row_exp, const int32_t *col_exp, int two_bits,
                            double *out, int64_t rows, int64_t cols, int n_mod) {
    crt_all(residues, 0, wh, wm, wl, M_hi, M_lo, inv_M, row_exp, col_exp, two_bits, out, rows,
            cols, n_mod);
}

void oracle_crt_reconstruct_u8(const uint8_t *residues, const double *wh, const double *wm,
                               const double *wl, double M_hi, double M_lo, double inv_M,
                               const int32_t *row_exp, const int32_t *col_exp, int two_bits,
                               double *out, int64_t rows, int64_t cols, int n_mod) {
    crt_all(0, residues, wh, wm, wl, M_hi, M_lo, inv_M, row_exp, col_exp, two_bits, out, rows,
            cols, n_mod);
}

/*
 * Floor-mod residues of scaled integers, ozaki.py:41-46:
 * out[k][e] = (int8)(x[e] mod p_k) with the result in [0, p_k).
 */
void oracle_residues(const int64_t *x, int64_t n, const int32_t *moduli, int n_mod,
                     int8_t *out) {
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < n; ++e) {
        for (int k = 0; k < n_mod; ++k) {
            int64_t r = x[e] % moduli[k];
            if (r < 0) r += moduli[k];
            out[(int64_t)k * n + e] = (int8_t)r;
        }
    }
}
