// gemm_kernel.cuh -- the per-modulus INT8 GEMMs of Ozaki scheme II as ONE
// persistent, warp-specialised tcgen05 kernel (replaces the reference's
// cuBLASLt strided-batched GEMM + mod_reduce + crt_kernel, crt_kernel.cu:6-146).
//
// Work: output tiles of kTileM x BN (256 x 256 for a CTA pair); a unit (CTA or
// pair) owns tiles round-robin and runs the full K loop once per (tile,
// modulus).  Default order, modulus-major: every unit sweeps its tiles for
// modulus 0, then 1, ..., with the units aligned at each pass boundary so the
// grid streams one residue plane at a time through L2 (optionally with the
// last two passes interleaved, see unit_at).  Tile-major (all moduli of a
// tile back to back) is the bounded-staging alternative.
//
// Roles (one CTA per SM):
//   warp 0, one thread   TMA producer: A and B residue tiles [128 x 128 B] and
//                        [BN x 128 B] (SWIZZLE_128B) into a STAGES-deep ring.
//   warp 1, one thread   MMA issuer: 4 x tcgen05.mma.kind::i8 (K = 32 each) per
//                        stage into an int32 accumulator in TMEM; NACC
//                        accumulator buffers let the epilogue drain one while
//                        the next modulus accumulates.  Warp 1 owns TMEM.
//   warps 2 .. 2+NEPI    epilogue: tcgen05.ld the accumulator (each warp reads
//                        its TMEM lane quadrant, warp % 4), reduce mod p_l, and
//                          mode 0: store raw int32 products     (parity tap)
//                          mode 1: store uint8 residues          (parity tap)
//                          mode 2: stage uint8 residues in this thread's slice
//                                  of the CTA's scratch; after the last modulus
//                                  run the CRT for the thread's row segment and
//                                  write FP64 C.
//
// Every wait is bounded (mbar_wait): on timeout the CTA records the error,
// raises a shared abort flag, drains its in-flight TMA loads and MMAs, frees
// TMEM and exits; its epilogue first writes NaN over every output tile it had
// not finished, so a timed-out product cannot pass for a result.  The pass
// alignment of the modulus-major schedule is a locality hint, not a
// dependency: a producer that waits there longer than align_budget_ns stops
// aligning (and makes every other CTA stop), with no error.  No TMA multicast
// is used.
#pragma once

#include "crt_kernels.cuh"

namespace fpemu {

constexpr int kBM = 128;       // tile rows (TMEM lanes)
constexpr int kBK = 128;       // K bytes per stage: one 128-byte swizzle row
constexpr int kUmmaK = 32;     // K of one tcgen05.mma kind::i8

template <int CG_, int BN_, int STAGES_, int NEPI_, int NACC_>
struct GemmCfg {
    static constexpr int CG = CG_;  // CTAs per MMA: 1, or 2 (a cluster pair, M = 256)
    static constexpr int BN = BN_, STAGES = STAGES_, NEPI = NEPI_, NACC = NACC_;
    static constexpr int kTileM = kBM * CG;        // output rows per tile (per pair)
    static constexpr int kBRows = BN / CG;         // B rows (N) this CTA stages
    static constexpr int kStageA = kBM * kBK;
    static constexpr int kStageB = kBRows * kBK;
    static constexpr int kTxBytes = CG * (kStageA + kStageB);  // landing on the leader's barrier
    static constexpr int kThreads = 32 * (2 + NEPI);
    static constexpr int kTmemCols = NACC * BN;
    static constexpr int kColGroups = NEPI / 4;    // epilogue warps per lane quadrant
    static constexpr int kCols = BN / kColGroups;  // accumulator columns per epilogue thread
    static constexpr int kChunks = kCols / 32;     // 32-column TMEM loads per thread
    static constexpr int kBarBytes = 8 * (2 * STAGES + 2 * NACC + 1) + 16;
    static constexpr int kSmemBytes = 1024 + STAGES * (kStageA + kStageB) + kBarBytes;
    static_assert(CG == 1 || CG == 2, "CTA group");
    static_assert(NEPI % 4 == 0 && kCols % 32 == 0, "epilogue split");
    static_assert(BN % (16 * CG) == 0 && BN >= 32 && BN <= 256, "UMMA N");
    static_assert(kTmemCols == 32 || kTmemCols == 64 || kTmemCols == 128 || kTmemCols == 256 ||
                      kTmemCols == 512,
                  "TMEM allocation must be a power of two in [32, 512]");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    // One staging slot (mode 2): one CTA's 128 x BN share of a tile, n_mod bytes per
    // output (each epilogue thread owns n_mod * kCols bytes of it).
    static int64_t slot_bytes(int n_mod) { return (int64_t)n_mod * kBM * BN; }
};

// Band rasterisation: tiles go down `band_rows` tile rows, then to the next
// column; bands follow each other down the matrix.  Consecutive tiles share
// A rows (a band's strips stay in L2 while its columns stream past).
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int band_rows, int& tm, int& tn) {
    const int per_band = band_rows * tiles_n;
    const int band = tile / per_band;
    const int r = tile - band * per_band;
    const int first = band * band_rows;
    const int rows = min(tiles_m - first, band_rows);
    tm = first + r % rows;
    tn = r / rows;
}

__device__ __forceinline__ uint32_t pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return a | (b << 8) | (c << 16) | (d << 24);
}

// C column of column j of this product: j itself, or -- for a product over
// columns gathered from several column blocks of C -- segment j / col_seg of
// width col_seg, col_seg_stride apart.
__device__ __forceinline__ int64_t out_col(const GemmParams& P, int j) {
    return P.col_seg > 0 ? (int64_t)(j / P.col_seg) * P.col_seg_stride + j % P.col_seg : (int64_t)j;
}

// Write one reconstructed value: the double result, or its round-to-nearest
// float when C is float32, then the optional per-column bias added in C's type
// -- the order of the reference's `matmul(...).to(dtype)` followed by `+ bias`.
__device__ __forceinline__ void store_c(const GemmParams& P, double* crow, int64_t row, int col, double v) {
    const int64_t oc = out_col(P, col);
    if (P.c_f32) {
        float f = __double2float_rn(v);
        if (P.bias) f = __fadd_rn(f, static_cast<const float*>(P.bias)[col]);
        reinterpret_cast<float*>(P.C)[row * P.ldc + oc] = f;
    } else {
        if (P.bias) v = __dadd_rn(v, static_cast<const double*>(P.bias)[col]);
        crow[oc] = v;
    }
}

// One kernel for both CTA-group sizes.  With CG = 2 the grid is made of
// 2-CTA clusters; a pair owns a 256 x BN output tile: each CTA stages its 128
// rows of A and its BN/2 rows of B, the leader (cluster rank 0) issues the
// M = 256 MMAs, and each CTA's epilogue drains its own 128 TMEM lanes.
template <class Cfg, int MODE>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    ozaki_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ GemmParams P) {
    constexpr int CG = Cfg::CG, BN = Cfg::BN, STAGES = Cfg::STAGES, NACC = Cfg::NACC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::kStageA;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::kStageB);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + NACC;
    uint64_t* drain = tempty + NACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;  // 0 = leader
    const int unit = blockIdx.x / CG;                         // pair (or CTA) index
    const int num_units = gridDim.x / CG;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int a = 0; a < NACC; ++a) {
            mbar_init(tfull + a, 1);
            mbar_init(tempty + a, CG * Cfg::NEPI);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc<CG>(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish<CG>();
    }
    tc_fence_before();
    if constexpr (CG == 2) cluster_sync();  // peers see initialised barriers before any TMA/arrive
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // This CTA (pair) owns tiles r = unit, unit + num_units, ... (in band-raster
    // order) and walks (tile, modulus) units in the order P.sched selects.  All
    // three roles generate the same sequence.
    //
    // Modulus-major, optionally with an interleaved tail (P.tail): the last two passes a =
    // n_mod-2 and b = n_mod-1 are merged as (0,a) (1,a) (0,b) (2,a) (1,b) ...
    // (T-1,a) (T-2,b) (T-1,b), so each tile's CRT epilogue (b, about twice its
    // MMA time in FP64 work) alternates with a light epilogue (a) instead of
    // all CRTs queueing behind the last pass's MMAs.  (i,a) still precedes
    // (i,b), whose CRT reads the plane staged at (i,a).
    const bool spread = P.sched == kSchedSpread;
    const int my_tiles = (P.num_tiles - unit + num_units - 1) / num_units;
    const int my_units = spread ? (int)(((int64_t)P.num_tiles * P.n_mod - unit + num_units - 1) / num_units)
                                : my_tiles * P.n_mod;
    const bool tail = P.sched != kSchedTileMajor && P.tail && P.n_mod >= 2;
    const int tail_base = (P.n_mod - 2) * my_tiles;
    auto unit_at = [&](int idx, int& tile, int& l) {
        if (spread) {  // global unit u = l * num_tiles + tile, dealt out round-robin
            const int64_t u = (int64_t)idx * num_units + unit;
            l = (int)(u / P.num_tiles);
            tile = (int)(u - (int64_t)l * P.num_tiles);
            return;
        }
        int i;
        if (P.sched == kSchedTileMajor) {
            i = idx / P.n_mod;
            l = idx - i * P.n_mod;
        } else if (tail && idx >= tail_base) {
            const int j = idx - tail_base;
            if (j == 0) { i = 0; l = P.n_mod - 2; }
            else if (j == 2 * my_tiles - 1) { i = my_tiles - 1; l = P.n_mod - 1; }
            else if (j & 1) { i = (j + 1) >> 1; l = P.n_mod - 2; }
            else { i = (j >> 1) - 1; l = P.n_mod - 1; }
        } else {
            l = idx / my_tiles;
            i = idx - l * my_tiles;
        }
        tile = i * num_units + unit;
    };

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int stage = 0, issued = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int idx = 0; ok && idx < my_units; ++idx) {
                int tile, l, tm, tn;
                unit_at(idx, tile, l);
                // Test hook: the producers of unit 0 stop delivering here, as a stalled
                // producer would, so the consumers' bounded waits run out.
                if (unit == 0 && idx == P.test_stall_idx) break;
                // (With the interleaved tail, pass b has no barrier of its own: it
                // runs inside the merged final phase that pass a's barrier opens.)
                if (P.pass_ctr != nullptr && l > 0 && idx == l * my_tiles && !(tail && l == P.n_mod - 1)) {
                    // Modulus-major: start pass l only when every CTA has issued all of
                    // pass l-1, so the whole grid streams one modulus plane at a time and
                    // its A band stays in L2 (pairs with one tile fewer would otherwise
                    // drift a unit further ahead every pass).  The grid is sized to the
                    // device's active-cluster limit, but CTAs are only co-resident if no
                    // other kernel holds SMs; nothing this CTA reads depends on another
                    // CTA, so after align_budget_ns it gives up aligning -- and raises
                    // the flag that makes every CTA give up -- instead of failing.
                    atomicAdd(P.pass_ctr + l, 1u);
                    const volatile unsigned int* c = P.pass_ctr + l;
                    volatile unsigned int* give_up = P.pass_ctr + kPassGiveUp;
                    const uint64_t t0 = global_ns();
                    while (*c < gridDim.x && *give_up == 0u) {
                        if (*abort_flag) { ok = false; break; }
                        if (global_ns() - t0 > P.align_budget_ns) { *give_up = 1u; break; }
                        __nanosleep(64);
                    }
                    if (!ok) break;
                }
                tile_coords(tile, P.tiles_m, P.tiles_n, P.band_rows, tm, tn);
                const int arow = tm * Cfg::kTileM + (int)rank * kBM;
                const int brow = tn * BN + (int)rank * Cfg::kBRows;
                for (int kb = 0; kb < P.num_kb; ++kb) {
                    if (*abort_flag) { ok = false; break; }
                    if (!mbar_wait(empty + stage, ph ^ 1u, P.budget_ns)) {
                        report_error(&g_device_error, FPEMU_ERR_TIMEOUT, kWaitEmpty, tile);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    if constexpr (CG == 1) {
                        mbar_arrive_expect_tx(full + stage, Cfg::kTxBytes);
                        tma_load_3d(sA + stage * Cfg::kStageA, &tmA, full + stage, kb * kBK, arow, l);
                        tma_load_3d(sB + stage * Cfg::kStageB, &tmB, full + stage, kb * kBK, brow, l);
                    } else {
                        // Both CTAs' bytes land on the leader's full barrier.
                        if (rank == 0) mbar_arrive_expect_tx(full + stage, Cfg::kTxBytes);
                        const uint32_t fb = mapa_shared(smem_u32(full + stage), 0);
                        tma_load_3d_pair(sA + stage * Cfg::kStageA, &tmA, fb, kb * kBK, arow, l);
                        tma_load_3d_pair(sB + stage * Cfg::kStageB, &tmB, fb, kb * kBK, brow, l);
                    }
                    ++issued;
                    if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                }
            }
            // Loads still in flight must land before shared memory goes away.  The
            // leader's full barriers count both CTAs' bytes; the peer is held by the
            // closing cluster barrier until the leader has drained.
            if (CG == 1 || rank == 0) {
                const int outstanding = issued < STAGES ? issued : STAGES;
                for (int i = 0; i < outstanding; ++i) {
                    if (--stage < 0) { stage = STAGES - 1; ph ^= 1u; }
                    if (!mbar_wait(full + stage, ph, P.budget_ns)) {
                        report_error(&g_device_error, FPEMU_ERR_TIMEOUT, kWaitDrainTma, stage);
                        *abort_flag = 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0 && rank == 0) {
            constexpr uint32_t kIdesc = idesc_i8(Cfg::kTileM, BN);
            int stage = 0, acc = 0;
            uint32_t ph = 0, aph = 0;
            bool ok = true;
            for (int idx = 0; ok && idx < my_units; ++idx) {
                if (*abort_flag) { ok = false; break; }
                if (!mbar_wait(tempty + acc, aph ^ 1u, P.budget_ns)) {
                    report_error(&g_device_error, FPEMU_ERR_TIMEOUT, kWaitTmemEmpty, idx);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < P.num_kb; ++kb) {
                    if (!mbar_wait(full + stage, ph, P.budget_ns)) {
                        report_error(&g_device_error, FPEMU_ERR_TIMEOUT, kWaitFull, idx);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * Cfg::kStageA);
                    const uint32_t b0 = smem_u32(sB + stage * Cfg::kStageB);
#pragma unroll
                    for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
                        mma_i8<CG>(d_tmem, smem_desc_k_sw128(a0 + kk * kUmmaK), smem_desc_k_sw128(b0 + kk * kUmmaK),
                                   kIdesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    mma_commit<CG>(empty + stage);  // frees the stage (in both CTAs) once done
                    if (++stage == STAGES) { stage = 0; ph ^= 1u; }
                }
                if (!ok) break;
                mma_commit<CG>(tfull + acc);  // accumulator complete (in both CTAs)
                if (++acc == NACC) { acc = 0; aph ^= 1u; }
            }
            // Every MMA issued above must finish before TMEM is released.
            mma_commit_local<CG>(drain);
            if (!mbar_wait(drain, 0, P.budget_ns)) {
                report_error(&g_device_error, FPEMU_ERR_TIMEOUT, kWaitDrainMma, 0);
                *abort_flag = 1;
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        constexpr int kChunks = Cfg::kChunks;
        const int ew = warp - 2;
        const int quad = warp & 3;  // TMEM lanes this warp may read: [32*quad, 32*quad + 32)
        const int cg = ew >> 2;     // which kCols-wide slice of the tile
        const int row_in_tile = (int)rank * kBM + quad * 32 + lane;
        // This thread's part of a staging slot: for modulus l and chunk c the 32
        // bytes at ((ew*n_mod + l)*kChunks + c)*1 KiB + lane*32 (a warp's stores
        // cover one contiguous KiB).  Only this thread reads them back.
        const int64_t thread_off = ((int64_t)ew * P.n_mod * kChunks * 32 + lane) * 32;
        int acc = 0;
        uint32_t aph = 0;
        bool ok = true;
        int idx = 0;
        for (; ok && idx < my_units; ++idx) {
            int tile, l, tm, tn;
            unit_at(idx, tile, l);
            tile_coords(tile, P.tiles_m, P.tiles_n, P.band_rows, tm, tn);
            const int64_t row = (int64_t)tm * Cfg::kTileM + row_in_tile;
            const int col0 = tn * BN + cg * Cfg::kCols;
            uint8_t* scr = nullptr;
            if (MODE == kModeCrt) {
                const int64_t slot = P.sched == kSchedTileMajor ? (int64_t)blockIdx.x : (int64_t)tile * CG + rank;
                scr = P.scratch + slot * P.scratch_slot + thread_off;
            }
            const bool last = (l == P.n_mod - 1);

            if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
            bool got = mbar_wait(tfull + acc, aph, P.budget_ns);
            got = __all_sync(0xffffffffu, got);
            if (!got) {
                if (lane == 0) report_error(&g_device_error, FPEMU_ERR_TIMEOUT, kWaitTmemFull, idx);
                *abort_flag = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t taddr =
                tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + cg * Cfg::kCols);
            const uint32_t p = P.mc.p[l], mg = P.mc.magic[l], sh = P.mc.shift[l];
#pragma unroll 1
            for (int c = 0; c < kChunks; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(taddr + (uint32_t)(c * 32), v);
                tmem_ld_wait();
                const int cb = col0 + c * 32;
                if (MODE == kModeRaw) {
                    if (row < P.m) {
                        int32_t* o = static_cast<int32_t*>(P.out) + ((int64_t)l * P.m + row) * P.n;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (cb + j < P.n) o[cb + j] = (int32_t)v[j];
                    }
                } else {
                    uint32_t w[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        w[q] = pack4(mod_small(v[4 * q], p, mg, sh), mod_small(v[4 * q + 1], p, mg, sh),
                                     mod_small(v[4 * q + 2], p, mg, sh), mod_small(v[4 * q + 3], p, mg, sh));
                    if (MODE == kModeResidue) {
                        if (row < P.m) {
                            uint8_t* o = static_cast<uint8_t*>(P.out) + ((int64_t)l * P.m + row) * P.n;
                            if (cb + 32 <= P.n && ((reinterpret_cast<uintptr_t>(o + cb) & 15) == 0)) {
                                reinterpret_cast<uint4*>(o + cb)[0] = make_uint4(w[0], w[1], w[2], w[3]);
                                reinterpret_cast<uint4*>(o + cb)[1] = make_uint4(w[4], w[5], w[6], w[7]);
                            } else {
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    if (cb + j < P.n) o[cb + j] = (uint8_t)(w[j >> 2] >> (8 * (j & 3)));
                            }
                        }
                    } else {
                        uint4* d = reinterpret_cast<uint4*>(scr + ((int64_t)l * kChunks + c) * 1024);
                        d[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        d[1] = make_uint4(w[4], w[5], w[6], w[7]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (CG == 1) mbar_arrive(tempty + acc);
                else mbar_arrive_cluster(mapa_shared(smem_u32(tempty + acc), 0));
            }
            if (++acc == NACC) { acc = 0; aph ^= 1u; }

            if (MODE == kModeCrt && last && row < P.m) {
                // CRT for this thread's row segment (kCols columns, 16 at a time),
                // from the residues it staged for every modulus.
                const int re = P.row_exp[row];
                double* crow = P.C + row * P.ldc;
#pragma unroll 1
                for (int h = 0; h < kChunks * 2; ++h) {
                    const int cb = col0 + h * 16;
                    if (cb < P.n) {
                        double hi[16], lo[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) { hi[j] = 0.0; lo[j] = 0.0; }
                        const uint8_t* src = scr + (int64_t)(h >> 1) * 1024 + (h & 1) * 16;
#pragma unroll 1
                        for (int m2 = 0; m2 < P.n_mod; ++m2) {
                            const uint4 q = *reinterpret_cast<const uint4*>(src + (int64_t)m2 * kChunks * 1024);
                            const double wh = P.cc.wh[m2], wm = P.cc.wm[m2], wl = P.cc.wl[m2];
                            const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                crt_step((double)((qq[j >> 2] >> (8 * (j & 3))) & 0xFFu), wh, wm, wl, hi[j], lo[j]);
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int col = cb + j;
                            if (col < P.n) {
                                const double v = crt_scale(crt_finish(hi[j], lo[j], P.cc), re, P.col_exp[col],
                                                           P.two_bits);
                                store_c(P, crow, row, col, v);
                            }
                        }
                    }
                }
            }
        }
        if (MODE == kModeResidue && idx < my_units) {
            // Aborted at unit idx: mark this thread's part of every unit it did not
            // write with 0xFF, which no residue can be (p <= 127); the CRT kernel
            // turns an output with such a residue into NaN.
#pragma unroll 1
            for (int j = idx; j < my_units; ++j) {
                int tile, l, tm, tn;
                unit_at(j, tile, l);
                tile_coords(tile, P.tiles_m, P.tiles_n, P.band_rows, tm, tn);
                const int64_t row = (int64_t)tm * Cfg::kTileM + row_in_tile;
                if (row >= P.m) continue;
                const int col0 = tn * BN + cg * Cfg::kCols;
                uint8_t* o = static_cast<uint8_t*>(P.out) + ((int64_t)l * P.m + row) * P.n;
#pragma unroll 1
                for (int c = 0; c < Cfg::kCols && col0 + c < P.n; ++c) o[col0 + c] = 0xFFu;
            }
        }
        if (MODE == kModeCrt && idx < my_units) {
            // Aborted at unit idx: every tile whose last modulus comes at or after
            // idx was not reconstructed.  Mark this thread's part of them NaN.
            const double qnan = __longlong_as_double(0x7FF8000000000000ll);
#pragma unroll 1
            for (int j = idx; j < my_units; ++j) {
                int tile, l, tm, tn;
                unit_at(j, tile, l);
                if (l != P.n_mod - 1) continue;
                tile_coords(tile, P.tiles_m, P.tiles_n, P.band_rows, tm, tn);
                const int64_t row = (int64_t)tm * Cfg::kTileM + row_in_tile;
                if (row >= P.m) continue;
                const int col0 = tn * BN + cg * Cfg::kCols;
#pragma unroll 1
                for (int c = 0; c < Cfg::kCols && col0 + c < P.n; ++c) {
                    const int64_t oc = out_col(P, col0 + c);
                    if (P.c_f32) reinterpret_cast<float*>(P.C)[row * P.ldc + oc] = __double2float_rn(qnan);
                    else P.C[row * P.ldc + oc] = qnan;
                }
            }
        }
    }

    // Teardown: every role is done in this CTA; with a pair, also wait for the
    // other CTA (the leader's MMAs read the peer's shared memory and write its
    // TMEM), then free TMEM.
    tc_fence_before();
    if constexpr (CG == 2) cluster_sync();
    else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<CG>(tmem_base, Cfg::kTmemCols);
    }
}

}  // namespace fpemu
