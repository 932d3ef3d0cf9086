// split_kernels.cuh -- the fused scale/split step (ozaki.py:32-46 of the
// reference): per row of an operand, the power-of-two exponent of its largest
// magnitude, the exact scaling to a 53-bit (or `bits`-bit) integer with
// round-half-even, and that integer's floor-mod residue for every modulus,
// written as int8 planes [n_mod][rows][res_ld] with K contiguous (the layout
// the GEMM's TMA loads want).
//
// Two kernels cover the operand layouts:
//   split_rows_kernel    K is the contiguous axis (A row-major, or B given as
//                        the transpose of a row-major W): 128-bit loads along K,
//                        a warp/CTA max-reduction, then residues.
//   split_strided_*      K is strided (B row-major [K,N]): a column-max pass
//                        with coalesced loads along N, then a tiled pass that
//                        transposes through shared memory.
#pragma once

#include "fpemu_device.cuh"

namespace fpemu {

// frexp exponent of max(m, 1e-300) from the bit pattern of m = max|x| (ozaki.py:34-35).
__device__ __forceinline__ int exp_from_maxbits(uint64_t mb) {
    if (mb >= 0x7FF0000000000000ull) return kNonFiniteExp;  // Inf or NaN in the row
    double m = __longlong_as_double((long long)mb);
    if (m < 1e-300) m = 1e-300;
    return (int)((__double_as_longlong(m) >> 52) & 0x7FF) - 1022;
}

// 2^t for t in [-1022, 1023], built from its bit pattern.
__device__ __forceinline__ double pow2(int t) {
    return __longlong_as_double((long long)(t + 1023) << 52);
}

// Scaled integer round_half_even(x * 2^s) as an integer-valued double, for s in
// [-1024+bits, 1049]: two exact power-of-two products, then rint (half to even).
// A product that underflows is below 2^-400 and rounds to 0 either way.
__device__ __forceinline__ double scale_round(double x, double f1, double f2) {
    return rint(__dmul_rn(__dmul_rn(x, f1), f2));
}

// Residues of an integer-valued double x (|x| <= 2^53), floor-mod semantics.
//
// Step 1, per prime group (products P < 2^27, contiguous ranges of the
// modulus list): q = floor(x * RN(1/P)) is floor(x/P) up to +-1, so
// r0 = fma(-q, P, x) is exact and lies in [-P, 2P); r0 + (2P + 2^52) is an
// integer in [2^52, 2^53) whose low 32 bits are y = r0 + 2P, with
// y == x (mod P) and P <= y < 4P < 2^29.  Four FP64 operations, no conversion.
// Step 2, per prime p of the group: y mod p by magic-number division
// (exact for y < 2^31), three integer operations.
struct ModTable {
    uint32_t p[kMaxModuli], magic[kMaxModuli], shift[kMaxModuli];
};

constexpr ModTable make_mod_table() {
    ModTable t{};
    for (int i = 0; i < kMaxModuli; ++i) {
        const uint32_t p = (uint32_t)kPrimes[i];
        uint32_t s = 0;
        while ((2u << s) <= p) ++s;
        t.p[i] = p;
        t.shift[i] = s;
        t.magic[i] = (uint32_t)(((1ull << (32 + s)) + p - 1) / p);
    }
    return t;
}

constexpr ModTable kModTable = make_mod_table();

constexpr int kNumGroups = 5;
constexpr int kGroupFirst[kNumGroups + 1] = {0, 8, 13, 17, 21, 25};

constexpr double group_product(int g) {
    double P = 1.0;
    for (int i = kGroupFirst[g]; i < kGroupFirst[g + 1]; ++i) P *= (double)kPrimes[i];
    return P;
}

template <int G>
__device__ __forceinline__ uint32_t group_rem(double x) {
    constexpr double P = group_product(G);
    static_assert(P < 134217728.0, "group product must stay below 2^27");
    constexpr double invP = 1.0 / P;
    constexpr double off = 2.0 * P + 4503599627370496.0;  // 2P + 2^52
    const double q = floor(__dmul_rn(x, invP));
    const double r0 = __fma_rn(-q, P, x);
    return (uint32_t)__double2loint(__dadd_rn(r0, off));
}

template <int L>
__device__ __forceinline__ uint32_t prime_rem(uint32_t y) {
    constexpr uint32_t p = kModTable.p[L], magic = kModTable.magic[L], shift = kModTable.shift[L];
    return y - (__umulhi(y, magic) >> shift) * p;
}

template <int L>
__device__ __forceinline__ void store_plane(const uint32_t (&y)[16], int8_t* dst, int64_t res_plane) {
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
        w[q] = prime_rem<L>(y[4 * q]) | (prime_rem<L>(y[4 * q + 1]) << 8) | (prime_rem<L>(y[4 * q + 2]) << 16) |
               (prime_rem<L>(y[4 * q + 3]) << 24);
    *reinterpret_cast<uint4*>(dst + (int64_t)L * res_plane) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <int G, int L>
__device__ __forceinline__ void store_group_planes(const uint32_t (&y)[16], int n_mod, int8_t* dst,
                                                   int64_t res_plane) {
    constexpr int end = kGroupFirst[G + 1];
    if constexpr (L < end) {
        if (L < n_mod) {
            store_plane<L>(y, dst, res_plane);
            store_group_planes<G, L + 1>(y, n_mod, dst, res_plane);
        }
    }
}

template <int G>
__device__ __forceinline__ void store_groups_from(const double (&x)[16], int n_mod, int8_t* dst,
                                                  int64_t res_plane) {
    if constexpr (G < kNumGroups) {
        constexpr int first = kGroupFirst[G];
        if (first < n_mod) {
            uint32_t y[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = group_rem<G>(x[j]);
            store_group_planes<G, first>(y, n_mod, dst, res_plane);
            store_groups_from<G + 1>(x, n_mod, dst, res_plane);
        }
    }
}

// Residues of 16 consecutive scaled elements for every modulus, stored as one
// 16-byte vector per plane.  `dst` is plane 0 of the chunk; planes are
// res_plane apart.
__device__ __forceinline__ void store_chunk_residues(const double (&x)[16], int n_mod, int8_t* dst,
                                                     int64_t res_plane) {
    store_groups_from<0>(x, n_mod, dst, res_plane);
}

// ---------------------------------------------------------------------------
// K contiguous.  GROUP threads (a multiple of 32, dividing blockDim) own one
// row; each thread walks chunks of 16 elements, stride GROUP chunks.
// VEC: the row start is 16-byte aligned, so chunks load as 8 x 16 bytes.
// ---------------------------------------------------------------------------

// This thread's share of max |x| over a row, as the bit pattern of the
// magnitude (monotone for non-negative doubles; NaN patterns sort above Inf).
template <int GROUP, bool VEC>
__device__ __forceinline__ unsigned long long row_maxbits_part(const double* x, int64_t k, int gt) {
    unsigned long long mb = 0;
    const int64_t nchunk = (k + 15) / 16;
    for (int64_t c = gt; c < nchunk; c += GROUP) {
        const int64_t t0 = c * 16;
        if (VEC && t0 + 16 <= k) {
            const double2* p2 = reinterpret_cast<const double2*>(x + t0);
            double2 d[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) d[j] = __ldg(p2 + j);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                mb = max(mb, (unsigned long long)__double_as_longlong(d[j].x) & 0x7FFFFFFFFFFFFFFFull);
                mb = max(mb, (unsigned long long)__double_as_longlong(d[j].y) & 0x7FFFFFFFFFFFFFFFull);
            }
        } else {
            for (int j = 0; j < 16 && t0 + j < k; ++j) {
                const double d = __ldg(x + t0 + j);
                mb = max(mb, (unsigned long long)__double_as_longlong(d) & 0x7FFFFFFFFFFFFFFFull);
            }
        }
    }
    return mb;
}

// Max over the GROUP threads of a row slot (g = the slot in this CTA); every
// thread of the CTA must call it (it synchronises the CTA when GROUP > 32).
template <int GROUP>
__device__ __forceinline__ unsigned long long row_max_reduce(unsigned long long mb, int g,
                                                             unsigned long long* red) {
    constexpr int kWarps = GROUP / 32;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    if (kWarps > 1) {
        if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = mb;
        __syncthreads();
        mb = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) mb = max(mb, red[g * kWarps + w]);
        __syncthreads();
    }
    return mb;
}

// Residues of one row whose exponent e is known: every chunk of the row, all
// moduli (columns k..res_ld-1 written as zero).
template <int GROUP, bool VEC>
__device__ __forceinline__ void row_residues(const SplitParams& P, const double* x, int64_t row, int e, int gt) {
    const bool finite = e != kNonFiniteExp;
    const int s = P.bits - e;
    const double f1 = pow2(s >> 1), f2 = pow2(s - (s >> 1));
    const int64_t nchunk_out = P.res_ld / 16;
    int8_t* out_row = P.res + row * P.res_ld;
    for (int64_t c = gt; c < nchunk_out; c += GROUP) {
        const int64_t t0 = c * 16;
        double v[16];
        if (finite && VEC && t0 + 16 <= P.k) {
            const double2* p2 = reinterpret_cast<const double2*>(x + t0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const double2 d = __ldg(p2 + j);
                v[2 * j] = scale_round(d.x, f1, f2);
                v[2 * j + 1] = scale_round(d.y, f1, f2);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                v[j] = (finite && t0 + j < P.k) ? scale_round(__ldg(x + t0 + j), f1, f2) : 0.0;
        }
        store_chunk_residues(v, P.n_mod, out_row + t0, P.res_plane);
    }
}

// Two passes per row in one kernel: the row maximum, then (re-reading the row,
// from L2 when it is still there) the residues.
template <int GROUP, bool VEC>
__global__ void __launch_bounds__(256) split_rows_kernel(const __grid_constant__ SplitParams P) {
    static_assert(GROUP % 32 == 0 && 256 % GROUP == 0, "bad group");
    constexpr int kRowsPerCta = 256 / GROUP;
    __shared__ unsigned long long red[256 / 32];
    const int g = threadIdx.x / GROUP;   // row slot in this CTA
    const int gt = threadIdx.x % GROUP;  // thread within the row group
    for (int64_t row0 = (int64_t)blockIdx.x * kRowsPerCta; row0 < P.rows;
         row0 += (int64_t)gridDim.x * kRowsPerCta) {
        const int64_t row = row0 + g;
        const bool live = row < P.rows;
        const double* x = P.X + (live ? row : 0) * P.s_row;
        unsigned long long mb = live ? row_maxbits_part<GROUP, VEC>(x, P.k, gt) : 0ull;
        mb = row_max_reduce<GROUP>(mb, g, red);
        if (!live) continue;
        const int e = exp_from_maxbits(mb);
        if (gt == 0) P.exps[row] = e;
        row_residues<GROUP, VEC>(P, x, row, e, gt);
    }
}

// The two passes as two kernels (FPEMU_SPLIT_ROWS=2): first every row's
// exponent (one read of the operand at full bandwidth), ...
template <int GROUP, bool VEC>
__global__ void __launch_bounds__(256) split_rowexp_kernel(const __grid_constant__ SplitParams P) {
    constexpr int kRowsPerCta = 256 / GROUP;
    __shared__ unsigned long long red[256 / 32];
    const int g = threadIdx.x / GROUP;
    const int gt = threadIdx.x % GROUP;
    for (int64_t row0 = (int64_t)blockIdx.x * kRowsPerCta; row0 < P.rows;
         row0 += (int64_t)gridDim.x * kRowsPerCta) {
        const int64_t row = row0 + g;
        const bool live = row < P.rows;
        unsigned long long mb = live ? row_maxbits_part<GROUP, VEC>(P.X + row * P.s_row, P.k, gt) : 0ull;
        mb = row_max_reduce<GROUP>(mb, g, red);
        if (live && gt == 0) P.exps[row] = exp_from_maxbits(mb);
    }
}

// ... then the residues from the exponents (a second read of the operand).
template <int GROUP, bool VEC>
__global__ void __launch_bounds__(256) split_rowres_kernel(const __grid_constant__ SplitParams P) {
    constexpr int kRowsPerCta = 256 / GROUP;
    const int g = threadIdx.x / GROUP;
    const int gt = threadIdx.x % GROUP;
    for (int64_t row0 = (int64_t)blockIdx.x * kRowsPerCta; row0 < P.rows;
         row0 += (int64_t)gridDim.x * kRowsPerCta) {
        const int64_t row = row0 + g;
        if (row < P.rows) row_residues<GROUP, VEC>(P, P.X + row * P.s_row, row, P.exps[row], gt);
    }
}

// ---------------------------------------------------------------------------
// K strided.  Pass 1: colmax[r] = max over t of |X[r, t]| (as bit patterns),
// threads along r (coalesced when s_row == 1), blocks along t; colmax must be
// zeroed first.
// ---------------------------------------------------------------------------
constexpr int kColmaxK = 256;

__global__ void __launch_bounds__(256) split_colmax_kernel(const __grid_constant__ SplitParams P,
                                                           unsigned long long* colmax) {
    const int64_t r = (int64_t)blockIdx.x * 256 + threadIdx.x;
    if (r >= P.rows) return;
    const int64_t t0 = (int64_t)blockIdx.y * kColmaxK;
    const int64_t t1 = min(t0 + (int64_t)kColmaxK, P.k);
    unsigned long long mb = 0;
    const double* x = P.X + r * P.s_row;
    for (int64_t t = t0; t < t1; ++t)
        mb = max(mb, (unsigned long long)__double_as_longlong(__ldg(x + t * P.s_k)) & 0x7FFFFFFFFFFFFFFFull);
    atomicMax(colmax + r, mb);
}

// Pass 2: a CTA takes 32 rows x 128 k, loads them through shared memory
// (coalesced along r), then each thread emits 16 consecutive k of one row.
constexpr int kTileR = 32;
constexpr int kTileK = 128;

__global__ void __launch_bounds__(256) split_strided_kernel(const __grid_constant__ SplitParams P) {
    // Element (t, r) sits at tile[t][r ^ swz(t)], swz(t) = 4 * ((t / 16) % 8), so the
    // compute phase (8 k-chunks x 4 rows per warp) hits every bank pair once per
    // wavefront, and the load phase (32 rows of one t) writes a permutation.
    __shared__ double tile[kTileK][kTileR];
    const int64_t r0 = (int64_t)blockIdx.x * kTileR;
    const int64_t k0 = (int64_t)blockIdx.y * kTileK;

    // Load: thread (tr = tid % 32, tk = tid / 32) reads rows r0+tr, k = k0+tk+8i.
    // All 16 loads are issued before the first shared-memory store, so a CTA
    // keeps its whole 32 KB tile in flight.
    {
        const int tr = threadIdx.x % kTileR;
        const int tk = threadIdx.x / kTileR;
        const int64_t r = r0 + tr;
        double v[kTileK / 8];
#pragma unroll
        for (int i = 0; i < kTileK / 8; ++i) {
            const int64_t t = k0 + tk + 8 * i;
            v[i] = (r < P.rows && t < P.k) ? __ldg(P.X + r * P.s_row + t * P.s_k) : 0.0;
        }
#pragma unroll
        for (int i = 0; i < kTileK / 8; ++i) {
            const int lt = tk + 8 * i;
            tile[lt][tr ^ (((lt >> 4) & 7) << 2)] = v[i];
        }
    }
    __syncthreads();

    // Compute: thread (r = tid / 8, kc = tid % 8) handles k0 + 16*kc .. +16 of row r0 + r.
    const int lr = threadIdx.x / 8;
    const int kc = threadIdx.x % 8;
    const int64_t row = r0 + lr;
    const int64_t t0 = k0 + 16 * kc;
    if (row < P.rows && t0 < P.res_ld) {
        const int e = exp_from_maxbits(P.colmax[row]);
        if (blockIdx.y == 0 && kc == 0) P.exps[row] = e;
        const bool finite = e != kNonFiniteExp;
        const int s = P.bits - e;
        const double f1 = pow2(s >> 1), f2 = pow2(s - (s >> 1));
        double v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
            v[j] = (finite && t0 + j < P.k) ? scale_round(tile[16 * kc + j][lr ^ ((kc & 7) << 2)], f1, f2) : 0.0;
        store_chunk_residues(v, P.n_mod, P.res + row * P.res_ld + t0, P.res_plane);
    }
}

}  // namespace fpemu
