// fpemu_device.cuh -- device-side building blocks for sm_100a: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM alloc / MMA / commit / load)
// and the per-modulus integer constants shared by the split and GEMM kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fpemu_internal.h"

namespace fpemu {

// ----------------------------------------------------------------------------
// Error reporting from device code.  A wait that runs out of time records the
// first failure here (code, role, block) and the kernel unwinds; the host
// reads it back with fpemu_device_error().  Nothing traps.
// ----------------------------------------------------------------------------
struct DeviceError {
    int code;    // FPEMU_ERR_TIMEOUT, ...
    int where;   // which wait gave up (see kWait*)
    int block;   // blockIdx.x of the first failing CTA
    int detail;  // role-specific (unit index, stage, ...)
};

enum : int {
    kWaitFull = 1,       // MMA warp waiting for a TMA stage
    kWaitEmpty = 2,      // producer waiting for a free stage
    kWaitTmemFull = 3,   // epilogue waiting for an accumulator
    kWaitTmemEmpty = 4,  // MMA warp waiting for the epilogue to drain TMEM
    kWaitDrainTma = 5,   // producer draining its loads at exit
    kWaitDrainMma = 6,   // MMA warp draining its MMAs at exit
};

// The first device-side failure on this device (one copy per device that loads
// the library); read and cleared by fpemu_device_error().
__device__ DeviceError g_device_error;

// Optional host-visible copy of the first failure: a pinned, mapped host
// DeviceError set up by fpemu_watch_errors() for this device (null until then).
// The host reads it without synchronising (fpemu_poll_error).
__device__ DeviceError* g_host_error;

__device__ __forceinline__ void report_error(DeviceError* err, int code, int where, int detail) {
    if (err != nullptr && atomicCAS(&err->code, 0, code) == 0) {
        err->where = where;
        err->block = (int)blockIdx.x;
        err->detail = detail;
        __threadfence();
        volatile DeviceError* h = g_host_error;
        if (h != nullptr) {
            h->where = where;
            h->block = (int)blockIdx.x;
            h->detail = detail;
            __threadfence_system();
            h->code = code;  // last: a non-zero code means the other fields are set
            __threadfence_system();
        }
    }
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete, giving up after
// `budget_ns` of wall time (checked every 256 polls).  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t budget_ns) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(a, parity)) return true;
        if ((i & 255u) == 0u && global_ns() - t0 > budget_ns) return false;
    }
}

// ----------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tile load global -> shared, completion counted on `bar` in bytes.
// c0 is the innermost (K, bytes) coordinate and is always a multiple of 128.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// ----------------------------------------------------------------------------
// Thread-block clusters (CTA pairs for the 2-SM MMA)
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier that may live in another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 3-D tile load into this CTA's shared memory whose completion is counted on
// the pair leader's mbarrier (`bar_cluster_addr`, a shared::cluster address).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                                                 int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// ----------------------------------------------------------------------------
// tcgen05
// ----------------------------------------------------------------------------
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    if constexpr (CG == 1)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                     "r"(ncols)
                     : "memory");
    else
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                     "r"(ncols)
                     : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
    if constexpr (CG == 1)
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    else
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    if constexpr (CG == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
    else
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32.  CG = 1: one CTA;
// CG = 2: the CTA pair (issued by the leader; A and B halves in each CTA's
// shared memory at the same offsets, D rows split across the two TMEMs).
template <int CG>
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    if constexpr (CG == 1)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
}

// Arrive once every tcgen05.mma issued so far by this thread is done: on `bar`
// in this CTA (CG = 1), or on `bar` in both CTAs of the pair (CG = 2).
template <int CG>
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    if constexpr (CG == 1)
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(bar))
                     : "memory");
    else
        asm volatile(
            "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                smem_u32(bar)),
            "h"((unsigned short)3)
            : "memory");
}

// Same, arriving only on `bar` in the issuing CTA (the leader's drain barrier).
template <int CG>
__device__ __forceinline__ void mma_commit_local(uint64_t* bar) {
    if constexpr (CG == 1)
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(bar))
                     : "memory");
    else
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(bar))
                     : "memory");
}

// 32 lanes x 32 consecutive columns of 32-bit values: thread t of the warp
// gets lane (base_lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major operand staged by TMA with
// SWIZZLE_128B: rows of 128 bytes, 8-row groups 1024 bytes apart.
//   [0,14) start >> 4 | [16,30) LBO >> 4 (=1, unused for swizzled K-major)
//   [32,46) SBO >> 4 (=64) | [46,48) version 1 | [61,64) layout 2 = SWIZZLE_128B
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor for kind::i8: D s32, A and B unsigned 8-bit (the
// residues are in [0, p) with p <= 127), both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4)                      // D format: S32
           | (0u << 7) | (0u << 10)       // A, B: unsigned 8-bit
           | ((uint32_t)(n >> 3) << 17)   // N >> 3
           | ((uint32_t)(m >> 4) << 24);  // M >> 4
}

// ----------------------------------------------------------------------------
// Exact division of small non-negative integers by a modulus p < 128.
// For n < 2^31 and s = floor(log2 p), m = ceil(2^(32+s) / p) < 2^32:
//   floor(n / p) == umulhi(n, m) >> s
// (the error term n*(m*p - 2^(32+s)) / (p*2^(32+s)) stays below 2^-(1+s) <= 1/p).
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t mod_small(uint32_t n, uint32_t p, uint32_t magic,
                                              uint32_t shift) {
    const uint32_t q = __umulhi(n, magic) >> shift;
    return n - q * p;
}

}  // namespace fpemu
