// fpemu_api.cu -- the C ABI of libfpemu.so (declared in include/fpemu.h).
//
// Host side of the Ozaki scheme II pipeline: modulus planning and CRT weights
// (exact integer arithmetic), workspace layout, TMA tensor maps, and the
// launches of the split, GEMM and CRT kernels.  Nothing here allocates device
// memory: the caller passes every buffer, including the workspace.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <algorithm>
#include <string>

#include "crt_kernels.cuh"
#include "gemm_kernel.cuh"
#include "split_kernels.cuh"

using namespace fpemu;

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

#define FPEMU_CUDA(expr)                                                                        \
    do {                                                                                        \
        cudaError_t e_ = (expr);                                                                \
        if (e_ != cudaSuccess) return fail(FPEMU_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
    } while (0)

#define FPEMU_TRY(expr)              \
    do {                             \
        int s_ = (expr);             \
        if (s_ != FPEMU_OK) return s_; \
    } while (0)

// GEMM configurations.  Main: CTA pairs (2-SM MMA, M = 256) on 256 x 256
// tiles, a 6-stage ring of 32 KB per CTA, 8 epilogue warps, 2 accumulators of
// 256 TMEM columns.  Single: one CTA per 128 x 256 tile, 4 stages of 48 KB
// (kept as an independent cross-check; FPEMU_GEMM_CTAS=1 selects it).
using MainCfg = GemmCfg<2, 256, 6, 8, 2>;
using SingleCfg = GemmCfg<1, 256, 4, 8, 2>;
static_assert(MainCfg::BN == SingleCfg::BN, "both configurations share the workspace layout");

struct DevInfo {
    int sms = 0;
    int major = 0, minor = 0;
};

int device_info(DevInfo* out) {
    static std::mutex mu;
    static DevInfo cache[64];
    static bool have[64] = {};
    int dev = 0;
    FPEMU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(FPEMU_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!have[dev]) {
        DevInfo d;
        FPEMU_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
        FPEMU_CUDA(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
        FPEMU_CUDA(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
        cache[dev] = d;
        have[dev] = true;
    }
    *out = cache[dev];
    if (out->major != 10 || out->minor != 0)
        return fail(FPEMU_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                    out->major, out->minor);
    return FPEMU_OK;
}

// Split of a K-contiguous operand: 1 = both passes in one kernel (the row is
// re-read from L2), 2 = an exponent kernel, then a residue kernel
// (FPEMU_SPLIT_ROWS).  Under mode 1, FPEMU_SPLIT_CTAS caps the CTAs per SM, and
// so the rows in flight whose second pass must find them in L2.
int split_rows_mode() {
    const char* s = getenv("FPEMU_SPLIT_ROWS");
    return (s && atoi(s) == 2) ? 2 : 1;
}

int split_rows_ctas_per_sm() {
    const char* s = getenv("FPEMU_SPLIT_CTAS");
    const int v = s ? atoi(s) : 64;
    return v < 1 ? 1 : (v > 64 ? 64 : v);
}

// Test hook of the failure-detection tests (FPEMU_TEST_STALL_UNIT=i): the TMA
// producers of the GEMM's first unit stop delivering at their unit i, so the
// consumers' bounded waits run out exactly as they would behind a stalled
// producer.  Read on every call; -1 (unset) disables it.
int test_stall_idx() {
    const char* s = getenv("FPEMU_TEST_STALL_UNIT");
    return s && *s ? atoi(s) : -1;
}

uint64_t wait_budget_ns() {
    static uint64_t v = [] {
        const char* s = getenv("FPEMU_WAIT_BUDGET_MS");
        long long ms = s ? atoll(s) : 2000;
        if (ms < 10) ms = 10;
        return (uint64_t)ms * 1000000ull;
    }();
    return v;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// 3-D map over int8 residues [n_mod][rows][res_ld] (K innermost), box
// [1][box_rows][128 B], SWIZZLE_128B.  Out-of-range K and rows read as zero.
int make_residue_map(CUtensorMap* map, const void* base, int64_t k, int64_t rows, int n_mod,
                     int64_t res_ld, int64_t res_plane, int box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(FPEMU_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows, (cuuint64_t)n_mod};
    cuuint64_t strides[2] = {(cuuint64_t)res_ld, (cuuint64_t)res_plane};
    cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(FPEMU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): k=%lld rows=%lld n_mod=%d ld=%lld",
                    (int)r, (long long)k, (long long)rows, n_mod, (long long)res_ld);
    return FPEMU_OK;
}

// ---------------------------------------------------------------- planning --

// Little-endian 32-bit limbs, enough for 2*k*2^(2*bits) and the product of 30 primes.
struct Big {
    uint32_t w[10] = {};
    void mul_small(uint32_t m) {
        uint64_t carry = 0;
        for (auto& x : w) {
            const uint64_t t = (uint64_t)x * m + carry;
            x = (uint32_t)t;
            carry = t >> 32;
        }
    }
    static int cmp(const Big& a, const Big& b) {
        for (int i = 9; i >= 0; --i)
            if (a.w[i] != b.w[i]) return a.w[i] < b.w[i] ? -1 : 1;
        return 0;
    }
};

int plan_moduli(int64_t k, int bits, int* n_mod) {
    if (k < 0 || bits < 1 || bits > 64) return fail(FPEMU_ERR_INVALID, "plan_moduli: k=%lld bits=%d", (long long)k, bits);
    // target = 2 * k * 2^(2*bits)
    Big target;
    const int sh = 2 * bits + 1;
    const unsigned __int128 kk = (unsigned __int128)(uint64_t)k;
    for (int i = 0; i < 10; ++i) {
        const int lo_bit = 32 * i - sh;  // bit of k that lands at limb i bit 0
        unsigned __int128 v;
        if (lo_bit >= 0) v = lo_bit >= 128 ? 0 : (kk >> lo_bit);
        else v = (-lo_bit) >= 128 ? 0 : (kk << (-lo_bit));
        target.w[i] = (uint32_t)v;
    }
    Big prod;
    prod.w[0] = 1;
    for (int i = 0; i < kNumPrimes; ++i) {
        prod.mul_small((uint32_t)kPrimes[i]);
        if (Big::cmp(prod, target) > 0) {
            *n_mod = i + 1;
            return FPEMU_OK;
        }
    }
    return fail(FPEMU_ERR_NO_MODULI, "not enough primes for inner dim %lld, bits %d", (long long)k, bits);
}

typedef unsigned __int128 u128;
typedef __int128 i128;

int crt_weights(int n_mod, CrtConsts* c) {
    if (n_mod < 1 || n_mod > kMaxModuli)
        return fail(FPEMU_ERR_UNSUPPORTED, "n_mod=%d outside [1, %d]", n_mod, kMaxModuli);
    u128 M = 1;
    for (int i = 0; i < n_mod; ++i) M *= (u128)kPrimes[i];  // < 2^127 for n_mod <= 25
    for (int i = 0; i < n_mod; ++i) {
        const uint32_t p = (uint32_t)kPrimes[i];
        const u128 Mi = M / p;
        const uint32_t a = (uint32_t)(Mi % p);
        uint32_t inv = 0;
        for (uint32_t t = 1; t < p; ++t)
            if ((a * t) % p == 1) { inv = t; break; }
        const u128 w = Mi * inv;  // < M
        const double hi = (double)w;
        const i128 r = (i128)w - (i128)hi;
        const double mid = (double)r;
        const double lo = (double)(r - (i128)mid);
        c->wh[i] = hi;
        c->wm[i] = mid;
        c->wl[i] = lo;
    }
    c->M_hi = (double)M;
    c->M_lo = (double)((i128)M - (i128)c->M_hi);
    c->inv_M = 1.0 / c->M_hi;
    return FPEMU_OK;
}

void mod_consts(int n_mod, ModConsts* mc) {
    memset(mc, 0, sizeof *mc);
    for (int i = 0; i < n_mod; ++i) {
        const uint32_t p = (uint32_t)kPrimes[i];
        uint32_t s = 0;
        while ((2u << s) <= p) ++s;  // floor(log2 p)
        const uint64_t num = 1ull << (32 + s);
        mc->p[i] = p;
        mc->shift[i] = s;
        mc->magic[i] = (uint32_t)((num + p - 1) / p);
        mc->c18[i] = (uint32_t)((1ull << 18) % p);
        mc->c36[i] = (uint32_t)((1ull << 36) % p);
        mc->kneg[i] = p << 24;
    }
}

int64_t max_k(int n_mod) {
    if (n_mod < 1 || n_mod > kMaxModuli) return 0;
    const int64_t pm = kPrimes[n_mod - 1] - 1;
    return (int64_t)2147483647 / (pm * pm);
}

// ------------------------------------------------------------- workspace --

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }
inline int64_t res_ld_for(int64_t k) { return ((k + 15) / 16) * 16; }

bool use_pairs() {
    const char* s = getenv("FPEMU_GEMM_CTAS");
    return !(s && atoi(s) == 1);
}

// Co-resident clusters of the pair kernel on this device (GPC shapes may leave
// some SMs unpaired); the persistent grid must not exceed what runs at once.
template <class Cfg, int MODE>
int max_active_units(const DevInfo& d) {
    auto kern = ozaki_gemm_kernel<Cfg, MODE>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) != cudaSuccess)
        return 0;
    if (Cfg::CG == 1) return d.sms;
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * d.sms);
    cfg.blockDim = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = Cfg::CG;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) return 0;
    return clusters;
}

// Launch units (CTAs, or CTA pairs) for an m x n problem (capacity cached per
// device): the fewest units that still finish the tiles in the fewest waves, so
// 64 tiles take 64 pairs rather than 74 (no slower: every unit does one tile per
// pass either way) and leave SMs free for kernels on other streams.
template <class Cfg>
int gemm_cap(const DevInfo& d) {
    static std::mutex mu;
    static int cache[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (cache[dev & 63] == 0) cache[dev & 63] = max_active_units<Cfg, kModeCrt>(d);
    return cache[dev & 63];
}

template <class Cfg>
int gemm_units(const DevInfo& d, int64_t m, int64_t n) {
    const int cap = gemm_cap<Cfg>(d);
    const int64_t tiles = ((m + Cfg::kTileM - 1) / Cfg::kTileM) * ((n + Cfg::BN - 1) / Cfg::BN);
    if (cap <= 0 || tiles <= 0) return 0;
    const int64_t waves = (tiles + cap - 1) / cap;
    return (int)((tiles + waves - 1) / waves);
}

// Tile rows per raster band (FPEMU_BAND_ROWS).  Default 8: with 256-row tiles and
// K = 16384 a band's A strips for one modulus are 32 MB, which stays resident in
// the L2 while the band's columns stream past; measured on B200 at n = 16384 the
// GEMM reads 115 GB from DRAM with 8, 138 GB with 16, 240 GB with 32 and 160 GB
// with 4 (too many B re-reads).
int band_rows() {
    const char* s = getenv("FPEMU_BAND_ROWS");
    const int v = s ? atoi(s) : 8;
    return v < 1 ? 1 : (v > 1024 ? 1024 : v);
}

// Interleaved final passes of the modulus-major schedule (FPEMU_GEMM_TAIL=1).  Off by
// default: measured on B200 it lowers the cycles of the last passes at n = 16384 but
// raises power (the FP64 CRT runs beside the MMAs), so under the 1 kW cap the clock
// drops and the product is 1 % slower; at m = 131072, k = n = 8192 it is 2.5 % slower.
int gemm_tail() {
    const char* s = getenv("FPEMU_GEMM_TAIL");
    return (s && atoi(s) == 1) ? 1 : 0;
}

// Schedule of the fused kernel: modulus-major unless FPEMU_GEMM_SCHED=tile.
int gemm_sched() {
    const char* s = getenv("FPEMU_GEMM_SCHED");
    return (s && strcmp(s, "tile") == 0) ? kSchedTileMajor : kSchedModulusMajor;
}

// Which form the fused GEMM + CRT stage takes for an m x n product:
//   0, fused: one kernel -- per-modulus GEMMs, mod and the CRT in the epilogue;
//   1, split: the residue GEMM with every (tile, modulus) unit dealt out to all
//      CTA pairs (kSchedSpread), the residues to the workspace, then the CRT
//      kernel over every SM.  When a product has few tiles per CTA pair, the
//      fused kernel leaves pairs idle and runs each tile's moduli and FP64 CRT
//      on one pair; the split form spreads both over the device.
// Auto: split when the product has fewer than kSplitTilesPerUnit tiles per CTA
// pair the device holds.  FPEMU_GEMM_PATH=fused|split forces one.  Measured on
// B200 (same inputs, identical results): the split form takes 0.27x the fused
// time at n = 1024, 0.78x at 2048 and 4096, 0.93x at 8192 (14 tiles per pair),
// 0.92-0.94x on the multi-GPU chunk shapes (2048-16384 x 2048 x 8192-16384),
// but 1.18x at n = 16384 (55 tiles per pair), where its CTA pairs, which do not
// align their modulus passes, drift apart and lose the L2 reuse.
constexpr int kSplitTilesPerUnit = 28;

int gemm_path(const DevInfo& d, int64_t m, int64_t n) {
    const char* s = getenv("FPEMU_GEMM_PATH");
    if (s && strcmp(s, "fused") == 0) return 0;
    if (s && strcmp(s, "split") == 0) return 1;
    const bool pairs = use_pairs();
    const int64_t tm = pairs ? MainCfg::kTileM : SingleCfg::kTileM;
    const int64_t tiles = ((m + tm - 1) / tm) * ((n + MainCfg::BN - 1) / MainCfg::BN);
    const int cap = pairs ? gemm_cap<MainCfg>(d) : gemm_cap<SingleCfg>(d);
    return (cap > 0 && tiles < (int64_t)kSplitTilesPerUnit * cap) ? 1 : 0;
}

template <class Cfg>
int64_t staging_slots(const DevInfo& d, int64_t m, int64_t n, int sched) {
    if (sched == kSchedTileMajor) return (int64_t)gemm_units<Cfg>(d, m, n) * Cfg::CG;  // one per CTA
    const int64_t tiles = ((m + Cfg::kTileM - 1) / Cfg::kTileM) * ((n + Cfg::BN - 1) / Cfg::BN);
    return tiles * Cfg::CG;  // one per CTA share of every tile
}

// Staging bytes of the fused kernel; covers both GEMM configurations (their
// slots are the same size: one CTA's 128 x 256 share of a tile).
size_t gemm_scratch_bytes(const DevInfo& d, int64_t m, int64_t n, int n_mod, int sched) {
    static_assert(MainCfg::kBRows * MainCfg::CG == SingleCfg::BN, "slot sizes agree");
    if (gemm_path(d, m, n) == 1) return align256((size_t)n_mod * (size_t)m * (size_t)n) + 256;  // residues
    const int64_t slots = std::max(staging_slots<MainCfg>(d, m, n, sched), staging_slots<SingleCfg>(d, m, n, sched));
    // Plus the per-pass counters of the modulus-major schedule, after the slots.
    return align256((size_t)slots * (size_t)MainCfg::slot_bytes(n_mod)) + 256;
}

size_t pass_ctr_offset(const DevInfo& d, int64_t m, int64_t n, int n_mod, int sched) {
    return gemm_scratch_bytes(d, m, n, n_mod, sched) - 256;
}

struct Layout {
    int64_t res_ld;
    size_t a_res, b_res, row_exp, col_exp, colmax, scratch, total;
};

Layout layout(const DevInfo& d, int64_t m, int64_t n, int64_t k, int n_mod) {
    Layout L;
    L.res_ld = res_ld_for(k);
    size_t off = 0;
    L.a_res = off; off += align256((size_t)n_mod * m * L.res_ld);
    L.b_res = off; off += align256((size_t)n_mod * n * L.res_ld);
    L.row_exp = off; off += align256((size_t)m * 4);
    L.col_exp = off; off += align256((size_t)n * 4);
    L.colmax = off; off += align256((size_t)(m > n ? m : n) * 8);
    L.scratch = off; off += gemm_scratch_bytes(d, m, n, n_mod, gemm_sched());
    L.total = off;
    return L;
}

// ---------------------------------------------------------------- launches --

int launch_split(const SplitParams& P, uint64_t* colmax, const DevInfo& d, cudaStream_t st) {
    if (P.rows == 0) return FPEMU_OK;
    if (P.s_k == 1) {
        const bool vec = (reinterpret_cast<uintptr_t>(P.X) % 16 == 0) && (P.s_row % 2 == 0 || P.rows == 1);
        const int group = P.k <= 512 ? 32 : P.k <= 2048 ? 64 : P.k <= 8192 ? 128 : 256;
        const int64_t rows_per_cta = 256 / group;
        int64_t grid = (P.rows + rows_per_cta - 1) / rows_per_cta;
        const int two = split_rows_mode() == 2;
        const int64_t cap = (int64_t)d.sms * (two ? 64 : split_rows_ctas_per_sm());
        if (grid > cap) grid = cap;
#define FPEMU_SPLIT_ROWS(G)                                                                      \
    do {                                                                                         \
        if (two) {                                                                               \
            if (vec) split_rowexp_kernel<G, true><<<(unsigned)grid, 256, 0, st>>>(P);            \
            else split_rowexp_kernel<G, false><<<(unsigned)grid, 256, 0, st>>>(P);               \
            if (vec) split_rowres_kernel<G, true><<<(unsigned)grid, 256, 0, st>>>(P);            \
            else split_rowres_kernel<G, false><<<(unsigned)grid, 256, 0, st>>>(P);               \
        } else {                                                                                 \
            if (vec) split_rows_kernel<G, true><<<(unsigned)grid, 256, 0, st>>>(P);              \
            else split_rows_kernel<G, false><<<(unsigned)grid, 256, 0, st>>>(P);                 \
        }                                                                                        \
    } while (0)
        switch (group) {
            case 32: FPEMU_SPLIT_ROWS(32); break;
            case 64: FPEMU_SPLIT_ROWS(64); break;
            case 128: FPEMU_SPLIT_ROWS(128); break;
            default: FPEMU_SPLIT_ROWS(256); break;
        }
#undef FPEMU_SPLIT_ROWS
    } else {
        if (colmax == nullptr) return fail(FPEMU_ERR_INVALID, "split: strided K needs colmax scratch");
        FPEMU_CUDA(cudaMemsetAsync(colmax, 0, (size_t)P.rows * 8, st));
        dim3 g1((unsigned)((P.rows + 255) / 256), (unsigned)((P.k + kColmaxK - 1) / kColmaxK));
        split_colmax_kernel<<<g1, 256, 0, st>>>(P, reinterpret_cast<unsigned long long*>(colmax));
        FPEMU_CUDA(cudaGetLastError());
        SplitParams Q = P;
        Q.colmax = colmax;
        dim3 g2((unsigned)((P.rows + kTileR - 1) / kTileR), (unsigned)((P.res_ld + kTileK - 1) / kTileK));
        split_strided_kernel<<<g2, 256, 0, st>>>(Q);
    }
    FPEMU_CUDA(cudaGetLastError());
    return FPEMU_OK;
}

template <class Cfg, int MODE>
int launch_gemm_cfg(GemmParams& P, const int8_t* a_res, const int8_t* b_res, int64_t res_ld,
                    int64_t res_plane_b, const DevInfo& d, cudaStream_t st, int max_ctas) {
    const int64_t m = P.m, n = P.n;
    const int64_t res_plane_a = m * res_ld;
    CUtensorMap ta, tb;
    FPEMU_TRY(make_residue_map(&ta, a_res, P.k, m, P.n_mod, res_ld, res_plane_a, kBM));
    FPEMU_TRY(make_residue_map(&tb, b_res, P.k, n, P.n_mod, res_ld, res_plane_b, Cfg::kBRows));
    P.num_kb = (int)((P.k + kBK - 1) / kBK);
    P.tiles_m = (int)((m + Cfg::kTileM - 1) / Cfg::kTileM);
    P.tiles_n = (int)((n + Cfg::BN - 1) / Cfg::BN);
    P.num_tiles = P.tiles_m * P.tiles_n;
    P.band_rows = band_rows();
    P.budget_ns = wait_budget_ns();
    // A producer normally waits at a pass boundary for at most about one tile's
    // K loop (tens of microseconds at k = 16384); past this it stops aligning.
    P.align_budget_ns = std::min<uint64_t>(P.budget_ns, 1000000ull + 20ull * (uint64_t)P.k);
    P.test_stall_idx = test_stall_idx();
    mod_consts(P.n_mod, &P.mc);
    int units = gemm_units<Cfg>(d, m, n);
    if (P.sched == kSchedSpread)  // every unit the device holds, up to one per (tile, modulus)
        units = (int)std::min<int64_t>(gemm_cap<Cfg>(d), (int64_t)P.num_tiles * P.n_mod);
    if (max_ctas > 0 && units > max_ctas / Cfg::CG) units = max_ctas / Cfg::CG;
    if (units < 1) return fail(FPEMU_ERR_CUDA, "GEMM kernel cannot be made resident on this device");
    auto kern = ozaki_gemm_kernel<Cfg, MODE>;
    FPEMU_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(units * Cfg::CG));
    cfg.blockDim = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = Cfg::CG;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = Cfg::CG > 1 ? 1 : 0;
    FPEMU_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, P));
    return FPEMU_OK;
}

template <int MODE>
int launch_gemm(GemmParams& P, const int8_t* a_res, const int8_t* b_res, int64_t res_ld, int64_t res_plane_b,
                const DevInfo& d, cudaStream_t st, int max_ctas = 0) {
    if (P.m == 0 || P.n == 0) return FPEMU_OK;
    if (res_plane_b < (int64_t)P.n * res_ld || res_plane_b % 16 != 0)
        return fail(FPEMU_ERR_INVALID, "b_res plane stride %lld must be >= n*res_ld and a multiple of 16",
                    (long long)res_plane_b);
    if (max_ctas > 0 && max_ctas < 2 && use_pairs())
        return fail(FPEMU_ERR_INVALID, "max_ctas=%d: the pair GEMM needs at least 2 CTAs", max_ctas);
    return use_pairs() ? launch_gemm_cfg<MainCfg, MODE>(P, a_res, b_res, res_ld, res_plane_b, d, st, max_ctas)
                       : launch_gemm_cfg<SingleCfg, MODE>(P, a_res, b_res, res_ld, res_plane_b, d, st, max_ctas);
}

// ---------------------------------------------- allocation-free staging --
//
// Staging area of fpemu_gemm_crt_noalloc, for callers that must not allocate
// device memory.  It is part of this library's device image: every GPU on
// which the library's kernels are loaded holds these 64 MiB until the process
// exits.  Host code only ever sees the symbol as a stand-in; the device
// address comes from cudaGetSymbolAddress, once per device.
constexpr size_t kNoAllocScratchBytes = (size_t)FPEMU_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

int noalloc_scratch(uint8_t** out) {
    static std::mutex mu;
    static uint8_t* addr[64] = {};
    int dev = 0;
    FPEMU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(FPEMU_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(FPEMU_ERR_CUDA, "cudaGetSymbolAddress(staging area) failed on device %d: %s", dev,
                        cudaGetErrorString(e));
        addr[dev] = static_cast<uint8_t*>(p);
    }
    *out = addr[dev];
    return FPEMU_OK;
}

// Host-visible mirrors of g_device_error, one per device: a pinned host block
// mapped into the device address space, its device address stored in
// g_host_error of that device.  Set up by fpemu_watch_errors (which allocates
// pinned host memory once per process; no device memory).
int host_error_slot(volatile DeviceError** out, bool create) {
    static std::mutex mu;
    static DeviceError* block = nullptr;
    static bool armed[64] = {};
    int dev = 0;
    FPEMU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(FPEMU_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!armed[dev]) {
        if (!create) {
            *out = nullptr;
            return FPEMU_OK;
        }
        if (block == nullptr) {
            void* p = nullptr;
            FPEMU_CUDA(cudaHostAlloc(&p, 64 * sizeof(DeviceError), cudaHostAllocMapped | cudaHostAllocPortable));
            memset(p, 0, 64 * sizeof(DeviceError));
            block = static_cast<DeviceError*>(p);
        }
        DeviceError* dptr = nullptr;
        FPEMU_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dptr), block + dev, 0));
        FPEMU_CUDA(cudaMemcpyToSymbol(g_host_error, &dptr, sizeof dptr));
        armed[dev] = true;
    }
    *out = block + dev;
    return FPEMU_OK;
}

int check_gemm_args(int64_t m, int64_t n, int64_t k, int n_mod, const void* a_res, const void* b_res,
                    int64_t res_ld) {
    if (m < 0 || n < 0 || k < 1) return fail(FPEMU_ERR_INVALID, "bad sizes m=%lld n=%lld k=%lld", (long long)m, (long long)n, (long long)k);
    if (n_mod < 1 || n_mod > kMaxModuli) return fail(FPEMU_ERR_UNSUPPORTED, "n_mod=%d outside [1, %d]", n_mod, kMaxModuli);
    if (k > max_k(n_mod))
        return fail(FPEMU_ERR_UNSUPPORTED, "k=%lld exceeds the exact int32 accumulation limit %lld for n_mod=%d",
                    (long long)k, (long long)max_k(n_mod), n_mod);
    if (m > 0x7FFFFFFFll || n > 0x7FFFFFFFll) return fail(FPEMU_ERR_UNSUPPORTED, "m or n beyond 2^31-1");
    if (res_ld < k || res_ld % 16 != 0) return fail(FPEMU_ERR_INVALID, "res_ld=%lld must be >= k and a multiple of 16", (long long)res_ld);
    if ((m > 0 && n > 0) && (a_res == nullptr || b_res == nullptr)) return fail(FPEMU_ERR_INVALID, "null residue pointer");
    if ((reinterpret_cast<uintptr_t>(a_res) | reinterpret_cast<uintptr_t>(b_res)) % 16 != 0)
        return fail(FPEMU_ERR_INVALID, "residue buffers must be 16-byte aligned");
    return FPEMU_OK;
}

// The standalone CRT kernel over the whole device (or max_ctas CTAs).
int launch_crt(const CrtParams& P, const DevInfo& d, cudaStream_t st, int max_ctas) {
    const int64_t work = P.m * ((P.n + 15) / 16);
    int64_t grid = (work + 255) / 256;
    int64_t cap = (int64_t)d.sms * 8;
    if (max_ctas > 0 && cap > max_ctas) cap = max_ctas;
    if (grid > cap) grid = cap;
    if (grid < 1) return FPEMU_OK;
    crt_kernel<<<(unsigned)grid, 256, 0, st>>>(P);
    FPEMU_CUDA(cudaGetLastError());
    return FPEMU_OK;
}

int bits_ok(int bits) {
    if (bits < 1 || bits > 53) return fail(FPEMU_ERR_INVALID, "bits=%d outside [1, 53]", bits);
    return FPEMU_OK;
}

int gemm_crt_impl(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t* a_res, const int8_t* b_res,
                  int64_t res_ld, int64_t b_res_plane, const int32_t* row_exp, const int32_t* col_exp, int bits,
                  void* C, int64_t ldc, int c_dtype, const void* bias, int col_seg, int64_t col_seg_stride,
                  int max_ctas, void* workspace, size_t workspace_bytes, void* stream);

}  // namespace

// ==================================================================== C ABI ==

extern "C" {

const char* fpemu_status_string(int status) {
    switch (status) {
        case FPEMU_OK: return "ok";
        case FPEMU_ERR_INVALID: return "invalid argument";
        case FPEMU_ERR_NO_MODULI: return "not enough primes";
        case FPEMU_ERR_UNSUPPORTED: return "unsupported problem";
        case FPEMU_ERR_WORKSPACE: return "workspace too small or misaligned";
        case FPEMU_ERR_CUDA: return "CUDA error";
        case FPEMU_ERR_TIMEOUT: return "device wait timed out";
        case FPEMU_ERR_NO_DEVICE: return "unsupported device";
        default: return "unknown status";
    }
}

const char* fpemu_last_error(void) { return t_last_error.c_str(); }

int fpemu_abi_version(void) { return FPEMU_ABI_VERSION; }

int fpemu_plan_moduli(int64_t k, int bits, int* n_mod, int32_t* moduli) {
    if (n_mod == nullptr) return fail(FPEMU_ERR_INVALID, "n_mod is null");
    FPEMU_TRY(plan_moduli(k, bits, n_mod));
    if (moduli)
        for (int i = 0; i < *n_mod; ++i) moduli[i] = kPrimes[i];
    return FPEMU_OK;
}

int fpemu_crt_weights(int n_mod, double* wh, double* wm, double* wl, double* M_hi, double* M_lo,
                      double* inv_M) {
    if (!wh || !wm || !wl || !M_hi || !M_lo || !inv_M) return fail(FPEMU_ERR_INVALID, "null output");
    CrtConsts c;
    FPEMU_TRY(crt_weights(n_mod, &c));
    for (int i = 0; i < n_mod; ++i) {
        wh[i] = c.wh[i];
        wm[i] = c.wm[i];
        wl[i] = c.wl[i];
    }
    *M_hi = c.M_hi;
    *M_lo = c.M_lo;
    *inv_M = c.inv_M;
    return FPEMU_OK;
}

int64_t fpemu_max_k(int n_mod) { return max_k(n_mod); }

size_t fpemu_gemm_workspace_size(int64_t m, int64_t n, int n_mod) {
    DevInfo d;
    if (device_info(&d) != FPEMU_OK || m < 0 || n < 0 || n_mod < 1 || n_mod > kMaxModuli) return 0;
    return gemm_scratch_bytes(d, m, n, n_mod, gemm_sched());
}

int fpemu_gemm_kernels(int64_t m, int64_t n) {
    DevInfo d;
    if (device_info(&d) != FPEMU_OK || m < 0 || n < 0) return 0;
    if (m == 0 || n == 0) return 0;
    return gemm_path(d, m, n) == 1 ? 2 : 1;
}

size_t fpemu_workspace_size(int64_t m, int64_t n, int64_t k, int n_mod) {
    DevInfo d;
    if (device_info(&d) != FPEMU_OK || m < 0 || n < 0 || k < 1 || n_mod < 1 || n_mod > kMaxModuli) return 0;
    return layout(d, m, n, k, n_mod).total;
}

int fpemu_split(int64_t rows, int64_t k, const double* X, int64_t s_row, int64_t s_k, int bits, int n_mod,
                int8_t* res, int64_t res_ld, int64_t res_plane, int32_t* exps, uint64_t* colmax_scratch,
                void* stream) {
    DevInfo d;
    FPEMU_TRY(device_info(&d));
    FPEMU_TRY(bits_ok(bits));
    if (rows < 0 || k < 1 || s_row < 0 || s_k < 0) return fail(FPEMU_ERR_INVALID, "split: bad sizes or strides");
    if (n_mod < 1 || n_mod > kMaxModuli) return fail(FPEMU_ERR_UNSUPPORTED, "n_mod=%d outside [1, %d]", n_mod, kMaxModuli);
    if (res_ld < k || res_ld % 16 != 0 || res_plane < rows * res_ld || res_plane % 16 != 0)
        return fail(FPEMU_ERR_INVALID, "split: res_ld must be a multiple of 16 >= k, res_plane >= rows*res_ld");
    if (rows > 0 && (!X || !res || !exps)) return fail(FPEMU_ERR_INVALID, "split: null pointer");
    if (reinterpret_cast<uintptr_t>(res) % 16 != 0) return fail(FPEMU_ERR_INVALID, "split: res not 16-byte aligned");
    SplitParams P;
    memset(&P, 0, sizeof P);
    P.X = X;
    P.rows = rows;
    P.k = k;
    P.s_row = s_row;
    P.s_k = s_k;
    P.res = res;
    P.res_ld = res_ld;
    P.res_plane = res_plane;
    P.exps = exps;
    P.bits = bits;
    P.n_mod = n_mod;
    mod_consts(n_mod, &P.mc);
    return launch_split(P, colmax_scratch, d, static_cast<cudaStream_t>(stream));
}

int fpemu_gemm_residues(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t* a_res, const int8_t* b_res,
                        int64_t res_ld, int mode, void* out, void* workspace, size_t workspace_bytes,
                        void* stream) {
    (void)workspace;
    (void)workspace_bytes;
    DevInfo d;
    FPEMU_TRY(device_info(&d));
    FPEMU_TRY(check_gemm_args(m, n, k, n_mod, a_res, b_res, res_ld));
    if (mode != 0 && mode != 1) return fail(FPEMU_ERR_INVALID, "mode must be 0 (raw) or 1 (residues)");
    if (m > 0 && n > 0 && out == nullptr) return fail(FPEMU_ERR_INVALID, "null output");
    GemmParams P;
    memset(&P, 0, sizeof P);
    P.m = (int)m;
    P.n = (int)n;
    P.k = (int)k;
    P.n_mod = n_mod;
    P.out = out;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return mode == 0 ? launch_gemm<kModeRaw>(P, a_res, b_res, res_ld, n * res_ld, d, st)
                     : launch_gemm<kModeResidue>(P, a_res, b_res, res_ld, n * res_ld, d, st);
}

int fpemu_crt_reconstruct(int64_t m, int64_t n, int n_mod, const uint8_t* res, const int32_t* row_exp,
                          const int32_t* col_exp, int bits, double* C, int64_t ldc, void* stream) {
    DevInfo d;
    FPEMU_TRY(device_info(&d));
    FPEMU_TRY(bits_ok(bits));
    if (m < 0 || n < 0 || ldc < n) return fail(FPEMU_ERR_INVALID, "crt: bad sizes");
    if (m == 0 || n == 0) return FPEMU_OK;
    if (!res || !row_exp || !col_exp || !C) return fail(FPEMU_ERR_INVALID, "crt: null pointer");
    CrtConsts cc;
    FPEMU_TRY(crt_weights(n_mod, &cc));
    CrtParams P;
    memset(&P, 0, sizeof P);
    P.res = res;
    P.m = m;
    P.n = n;
    P.n_mod = n_mod;
    P.row_exp = row_exp;
    P.col_exp = col_exp;
    P.two_bits = 2 * bits;
    P.C = C;
    P.ldc = ldc;
    P.cc = cc;
    return launch_crt(P, d, static_cast<cudaStream_t>(stream), 0);
}

int fpemu_gemm_crt(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t* a_res, const int8_t* b_res,
                   int64_t res_ld, int64_t b_res_plane, const int32_t* row_exp, const int32_t* col_exp, int bits,
                   double* C, int64_t ldc, int max_ctas, void* workspace, size_t workspace_bytes, void* stream) {
    return fpemu_gemm_crt_ex(m, n, k, n_mod, a_res, b_res, res_ld, b_res_plane, row_exp, col_exp, bits, C, ldc,
                             FPEMU_C_F64, nullptr, max_ctas, workspace, workspace_bytes, stream);
}

int fpemu_gemm_crt_ex(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t* a_res, const int8_t* b_res,
                      int64_t res_ld, int64_t b_res_plane, const int32_t* row_exp, const int32_t* col_exp, int bits,
                      void* C, int64_t ldc, int c_dtype, const void* bias, int max_ctas, void* workspace,
                      size_t workspace_bytes, void* stream) {
    return gemm_crt_impl(m, n, k, n_mod, a_res, b_res, res_ld, b_res_plane, row_exp, col_exp, bits, C, ldc, c_dtype,
                         bias, 0, 0, max_ctas, workspace, workspace_bytes, stream);
}

int fpemu_gemm_crt_segmented(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t* a_res, const int8_t* b_res,
                             int64_t res_ld, int64_t b_res_plane, const int32_t* row_exp, const int32_t* col_exp,
                             int bits, double* C, int64_t ldc, int64_t col_seg, int64_t col_seg_stride, int max_ctas,
                             void* workspace, size_t workspace_bytes, void* stream) {
    if (col_seg < 1 || col_seg > 0x7FFFFFFFll || col_seg_stride < col_seg)
        return fail(FPEMU_ERR_INVALID, "gemm_crt_segmented: col_seg=%lld, col_seg_stride=%lld (need 1 <= col_seg <= "
                    "col_seg_stride)", (long long)col_seg, (long long)col_seg_stride);
    if (n > 0 && ((n - 1) / col_seg) * col_seg_stride + (n - 1) % col_seg >= ldc)
        return fail(FPEMU_ERR_INVALID, "gemm_crt_segmented: the last column lands past ldc=%lld", (long long)ldc);
    return gemm_crt_impl(m, n, k, n_mod, a_res, b_res, res_ld, b_res_plane, row_exp, col_exp, bits, C, ldc,
                         FPEMU_C_F64, nullptr, (int)col_seg, col_seg_stride, max_ctas, workspace, workspace_bytes,
                         stream);
}

}  // extern "C"

namespace {

int gemm_crt_impl(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t* a_res, const int8_t* b_res,
                  int64_t res_ld, int64_t b_res_plane, const int32_t* row_exp, const int32_t* col_exp, int bits,
                  void* C, int64_t ldc, int c_dtype, const void* bias, int col_seg, int64_t col_seg_stride,
                  int max_ctas, void* workspace, size_t workspace_bytes, void* stream) {
    if (c_dtype != FPEMU_C_F64 && c_dtype != FPEMU_C_F32)
        return fail(FPEMU_ERR_INVALID, "c_dtype=%d: expected FPEMU_C_F64 (0) or FPEMU_C_F32 (1)", c_dtype);
    if (bias != nullptr && reinterpret_cast<uintptr_t>(bias) % (c_dtype == FPEMU_C_F32 ? 4 : 8) != 0)
        return fail(FPEMU_ERR_INVALID, "bias is not aligned to its element size");
    DevInfo d;
    FPEMU_TRY(device_info(&d));
    FPEMU_TRY(bits_ok(bits));
    FPEMU_TRY(check_gemm_args(m, n, k, n_mod, a_res, b_res, res_ld));
    if (m == 0 || n == 0) return FPEMU_OK;
    if (!row_exp || !col_exp || !C || ldc < n) return fail(FPEMU_ERR_INVALID, "gemm_crt: bad output arguments");
    const int sched = gemm_sched();
    const size_t need = gemm_scratch_bytes(d, m, n, n_mod, sched);
    if (workspace == nullptr || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(FPEMU_ERR_WORKSPACE, "gemm_crt: need %zu bytes of 256-byte aligned workspace, got %zu",
                    need, workspace_bytes);
    if (gemm_path(d, m, n) == 1) {
        // Split form: spread residue GEMM into the workspace, then the CRT kernel.
        GemmParams G;
        memset(&G, 0, sizeof G);
        G.m = (int)m;
        G.n = (int)n;
        G.k = (int)k;
        G.n_mod = n_mod;
        G.out = workspace;
        G.sched = kSchedSpread;
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        FPEMU_TRY(launch_gemm<kModeResidue>(G, a_res, b_res, res_ld, b_res_plane, d, st, max_ctas));
        CrtParams Q;
        memset(&Q, 0, sizeof Q);
        Q.res = static_cast<const uint8_t*>(workspace);
        Q.m = m;
        Q.n = n;
        Q.n_mod = n_mod;
        Q.row_exp = row_exp;
        Q.col_exp = col_exp;
        Q.two_bits = 2 * bits;
        Q.C = C;
        Q.ldc = ldc;
        Q.c_f32 = c_dtype == FPEMU_C_F32;
        Q.bias = bias;
        Q.col_seg = col_seg;
        Q.col_seg_stride = col_seg_stride;
        FPEMU_TRY(crt_weights(n_mod, &Q.cc));
        return launch_crt(Q, d, st, max_ctas);
    }
    GemmParams P;
    memset(&P, 0, sizeof P);
    P.m = (int)m;
    P.n = (int)n;
    P.k = (int)k;
    P.n_mod = n_mod;
    P.C = static_cast<double*>(C);
    P.ldc = ldc;
    P.bias = bias;
    P.c_f32 = c_dtype == FPEMU_C_F32;
    P.col_seg = col_seg;
    P.col_seg_stride = col_seg_stride;
    P.row_exp = row_exp;
    P.col_exp = col_exp;
    P.two_bits = 2 * bits;
    P.scratch = static_cast<uint8_t*>(workspace);
    P.scratch_slot = MainCfg::slot_bytes(n_mod);
    P.sched = sched;
    P.tail = gemm_tail();
    if (sched == kSchedModulusMajor) {
        P.pass_ctr = reinterpret_cast<unsigned int*>(P.scratch + pass_ctr_offset(d, m, n, n_mod, sched));
        FPEMU_CUDA(cudaMemsetAsync(P.pass_ctr, 0, 256, static_cast<cudaStream_t>(stream)));
    }
    FPEMU_TRY(crt_weights(n_mod, &P.cc));
    return launch_gemm<kModeCrt>(P, a_res, b_res, res_ld, b_res_plane, d, static_cast<cudaStream_t>(stream),
                                 max_ctas);
}

}  // namespace

extern "C" {

int fpemu_gemm_crt_noalloc(int64_t m, int64_t n, int64_t k, int n_mod, const int8_t* a_res,
                           const int8_t* b_res, int64_t res_ld, const int32_t* row_exp,
                           const int32_t* col_exp, int bits, double* C, int64_t ldc, void* stream) {
    DevInfo d;
    FPEMU_TRY(device_info(&d));
    FPEMU_TRY(bits_ok(bits));
    FPEMU_TRY(check_gemm_args(m, n, k, n_mod, a_res, b_res, res_ld));
    if (m == 0 || n == 0) return FPEMU_OK;
    if (!row_exp || !col_exp || !C || ldc < n)
        return fail(FPEMU_ERR_INVALID, "gemm_crt_noalloc: bad output arguments");
    // Each CTA stages n_mod * 128 * 256 bytes; the grid shrinks to what the
    // static area holds, and a modulus count that cannot fit one CTA pair is refused.
    const int64_t per_cta = MainCfg::slot_bytes(n_mod);
    const int64_t fit = (int64_t)kNoAllocScratchBytes / per_cta;
    if (fit < 2)
        return fail(FPEMU_ERR_WORKSPACE,
                    "gemm_crt_noalloc: n_mod=%d needs %lld bytes per CTA pair, more than the %zu-byte static "
                    "staging area", n_mod, (long long)(2 * per_cta), kNoAllocScratchBytes);
    uint8_t* scratch = nullptr;
    FPEMU_TRY(noalloc_scratch(&scratch));
    GemmParams P;
    memset(&P, 0, sizeof P);
    P.m = (int)m;
    P.n = (int)n;
    P.k = (int)k;
    P.n_mod = n_mod;
    P.C = C;
    P.ldc = ldc;
    P.row_exp = row_exp;
    P.col_exp = col_exp;
    P.two_bits = 2 * bits;
    P.scratch = scratch;
    P.scratch_slot = per_cta;
    P.sched = kSchedTileMajor;  // one reusable slot per CTA: bounded staging
    FPEMU_TRY(crt_weights(n_mod, &P.cc));
    const int max_ctas = (int)std::min<int64_t>(fit & ~(int64_t)1, 1 << 20);
    return launch_gemm<kModeCrt>(P, a_res, b_res, res_ld, n * res_ld, d, static_cast<cudaStream_t>(stream),
                                 max_ctas);
}

int fpemu_ozaki2_dgemm(int64_t m, int64_t n, int64_t k, const double* A, int64_t sA_row, int64_t sA_col,
                       const double* B, int64_t sB_row, int64_t sB_col, double* C, int64_t ldc, int bits,
                       int n_mod, void* workspace, size_t workspace_bytes, void* stream) {
    return fpemu_ozaki2_gemm_ex(m, n, k, A, sA_row, sA_col, B, sB_row, sB_col, C, ldc, FPEMU_C_F64, nullptr, bits,
                                n_mod, workspace, workspace_bytes, stream);
}

int fpemu_ozaki2_gemm_ex(int64_t m, int64_t n, int64_t k, const double* A, int64_t sA_row, int64_t sA_col,
                         const double* B, int64_t sB_row, int64_t sB_col, void* C, int64_t ldc, int c_dtype,
                         const void* bias, int bits, int n_mod, void* workspace, size_t workspace_bytes,
                         void* stream) {
    DevInfo d;
    FPEMU_TRY(device_info(&d));
    FPEMU_TRY(bits_ok(bits));
    if (m < 0 || n < 0 || k < 1) return fail(FPEMU_ERR_INVALID, "bad sizes m=%lld n=%lld k=%lld", (long long)m, (long long)n, (long long)k);
    if (sA_row < 0 || sA_col < 0 || sB_row < 0 || sB_col < 0 || ldc < n)
        return fail(FPEMU_ERR_INVALID, "negative stride or ldc < n");
    if (m == 0 || n == 0) return FPEMU_OK;
    if (!A || !B || !C) return fail(FPEMU_ERR_INVALID, "null matrix pointer");
    if (n_mod == 0) FPEMU_TRY(plan_moduli(k, bits, &n_mod));
    if (n_mod < 1 || n_mod > kMaxModuli) return fail(FPEMU_ERR_UNSUPPORTED, "n_mod=%d outside [1, %d]", n_mod, kMaxModuli);
    if (k > max_k(n_mod))
        return fail(FPEMU_ERR_UNSUPPORTED, "k=%lld exceeds the exact int32 accumulation limit %lld",
                    (long long)k, (long long)max_k(n_mod));
    const Layout L = layout(d, m, n, k, n_mod);
    if (workspace == nullptr || workspace_bytes < L.total || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
        return fail(FPEMU_ERR_WORKSPACE, "need %zu bytes of 256-byte aligned workspace, got %zu", L.total,
                    workspace_bytes);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int8_t* a_res = reinterpret_cast<int8_t*>(ws + L.a_res);
    int8_t* b_res = reinterpret_cast<int8_t*>(ws + L.b_res);
    int32_t* re = reinterpret_cast<int32_t*>(ws + L.row_exp);
    int32_t* ce = reinterpret_cast<int32_t*>(ws + L.col_exp);
    uint64_t* colmax = reinterpret_cast<uint64_t*>(ws + L.colmax);
    FPEMU_TRY(fpemu_split(m, k, A, sA_row, sA_col, bits, n_mod, a_res, L.res_ld, m * L.res_ld, re, colmax, stream));
    FPEMU_TRY(fpemu_split(n, k, B, sB_col, sB_row, bits, n_mod, b_res, L.res_ld, n * L.res_ld, ce, colmax, stream));
    return fpemu_gemm_crt_ex(m, n, k, n_mod, a_res, b_res, L.res_ld, n * L.res_ld, re, ce, bits, C, ldc, c_dtype,
                             bias, 0, ws + L.scratch, L.total - L.scratch, stream);
}

int fpemu_device_error(int* code, int* where, int* block, int* detail, int clear) {
    if (code == nullptr) return fail(FPEMU_ERR_INVALID, "code is null");
    FPEMU_CUDA(cudaDeviceSynchronize());
    DeviceError e;
    FPEMU_CUDA(cudaMemcpyFromSymbol(&e, g_device_error, sizeof e));
    *code = e.code;
    if (where) *where = e.where;
    if (block) *block = e.block;
    if (detail) *detail = e.detail;
    if (clear) {
        DeviceError z;
        memset(&z, 0, sizeof z);
        FPEMU_CUDA(cudaMemcpyToSymbol(g_device_error, &z, sizeof z));
        volatile DeviceError* h = nullptr;
        FPEMU_TRY(host_error_slot(&h, false));
        if (h != nullptr) h->code = 0;
    }
    return FPEMU_OK;
}

int fpemu_watch_errors(void) {
    volatile DeviceError* h = nullptr;
    return host_error_slot(&h, true);
}

int fpemu_poll_error(int* code, int* where, int* block, int* detail) {
    if (code == nullptr) return fail(FPEMU_ERR_INVALID, "code is null");
    volatile DeviceError* h = nullptr;
    FPEMU_TRY(host_error_slot(&h, false));
    if (h == nullptr) return fail(FPEMU_ERR_INVALID, "fpemu_poll_error: fpemu_watch_errors was not called on this device");
    *code = h->code;
    if (where) *where = h->where;
    if (block) *block = h->block;
    if (detail) *detail = h->detail;
    return FPEMU_OK;
}

}  // extern "C"
