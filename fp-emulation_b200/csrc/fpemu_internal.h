// fpemu_internal.h -- structures shared by the host API and the kernels.
#pragma once

#include <stdint.h>

#include "../../include/fpemu.h"

namespace fpemu {

constexpr int kMaxModuli = 25;  // 25 primes cover k <= 214748 at 53 bits (int32 limit)
constexpr int kNumPrimes = 30;
constexpr int kPrimes[kNumPrimes] = {3,  5,  7,  11, 13, 17, 19, 23, 29, 31,  37,  41,  43,  47,  53,
                                     59, 61, 67, 71, 73, 79, 83, 89, 97, 101, 103, 107, 109, 113, 127};

// Row/column exponent recorded for a row or column that holds NaN or +-Inf;
// every output element that depends on it becomes NaN.
constexpr int kNonFiniteExp = -0x40000000;

// Per-modulus integer constants (see mod_small in fpemu_device.cuh).
struct ModConsts {
    uint32_t p[kMaxModuli];
    uint32_t magic[kMaxModuli];
    uint32_t shift[kMaxModuli];
    uint32_t c18[kMaxModuli];
    uint32_t c36[kMaxModuli];
    uint32_t kneg[kMaxModuli];
};

// CRT constants, ozaki.py:62-80.
struct CrtConsts {
    double wh[kMaxModuli];
    double wm[kMaxModuli];
    double wl[kMaxModuli];
    double M_hi, M_lo, inv_M;
};

// The standalone CRT kernel: C from uint8 residues [n_mod][m][n], with the
// output options of the fused epilogue (float32 cast, bias, column segments).
struct CrtParams {
    const uint8_t* res;
    int64_t m, n;
    int n_mod;
    const int32_t* row_exp;
    const int32_t* col_exp;
    int two_bits;
    void* C;
    int64_t ldc;
    int c_f32;
    const void* bias;
    int col_seg;
    int64_t col_seg_stride;
    CrtConsts cc;
};

struct SplitParams {
    const double* X;
    int64_t rows, k, s_row, s_k;
    int8_t* res;
    int64_t res_ld, res_plane;
    int32_t* exps;
    const uint64_t* colmax;  // strided variant only
    int bits, n_mod;
    ModConsts mc;
};

enum GemmMode : int { kModeRaw = 0, kModeResidue = 1, kModeCrt = 2 };

// Order in which a CTA (pair) walks its (tile, modulus) units.
//   kSchedModulusMajor: every CTA owns a fixed set of tiles and sweeps them once per
//     modulus, so at any time all CTAs read the same modulus plane of A and B
//     (L2 reuse as in one plain GEMM); residues are staged per tile (workspace
//     n_mod bytes per output element).
//   kSchedTileMajor: all moduli of a tile back to back; staging is one reusable
//     slot per CTA (bounded workspace), at the cost of re-reading A and B strips
//     from DRAM for every modulus.
//   kSchedSpread (mode 1 only, the split path): the (tile, modulus) units of the
//     whole product are dealt out round-robin in modulus-major order to every
//     CTA (pair), so a product with fewer tiles than CTAs still uses them all;
//     the residues go to global memory and a separate kernel runs the CRT.
enum GemmSched : int { kSchedModulusMajor = 0, kSchedTileMajor = 1, kSchedSpread = 2 };

// Index of the "stop aligning" flag in the 64 pass counters of the modulus-major
// schedule (passes use [0, n_mod), n_mod <= 25).
constexpr int kPassGiveUp = 63;

struct GemmParams {
    int m, n, k, n_mod;
    int num_kb;            // ceil(k / 128)
    int tiles_m, tiles_n, num_tiles;
    int band_rows;         // tile rows per raster band
    void* out;             // raw int32 / uint8 residues, [n_mod][m][n] (modes 0, 1)
    double* C;             // mode 2 (float* when c_f32)
    int64_t ldc;
    const void* bias;      // mode 2, optional: per-column bias in C's type, added after the cast
    int c_f32;             // mode 2: C is float (the double result rounded to nearest)
    int col_seg;           // mode 2: > 0 scatters column j of this product to C column
    int64_t col_seg_stride;  //   (j / col_seg) * col_seg_stride + j % col_seg; 0 keeps column j
    const int32_t* row_exp;
    const int32_t* col_exp;
    int two_bits;
    uint8_t* scratch;      // mode 2: residue staging
    int64_t scratch_slot;  // bytes of one staging slot (one CTA's share of one tile)
    int sched;             // GemmSched
    int tail;              // modulus-major: interleave the last two passes (CRT next to light epilogues)
    unsigned int* pass_ctr;  // modulus-major: zeroed counters aligning the producers per pass
                             // ([l] for pass l; [kPassGiveUp] set when alignment is abandoned)
    uint64_t budget_ns;    // bound on every mbarrier wait
    uint64_t align_budget_ns;  // how long a producer waits at a pass boundary before it stops aligning
    int test_stall_idx;    // test hook (-1 = off): unit 0's producers issue nothing from this unit on
    ModConsts mc;
    CrtConsts cc;
};

}  // namespace fpemu
