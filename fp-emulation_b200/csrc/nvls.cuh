// nvls.cuh -- NVLink multicast (NVLS) stores and the cross-GPU progress
// counters of the multi-GPU product.
//
// A multicast address (an NVLS object bound to one buffer on every GPU of the
// group) takes `multimem.st`: the NVSwitch writes the value into every GPU's
// copy, so a split kernel that stores its residues there broadcasts them with
// one NVLink egress.  Ordering between GPUs uses monotonically growing 64-bit
// counters: a producer adds to a counter with release semantics at system scope
// after its stores; a consumer's stream runs a one-thread kernel that polls the
// counter with acquire loads until it reaches a target, so the kernels after it
// in the stream see the producer's data.  Every poll is bounded in time: on
// expiry the wait records FPEMU_ERR_TIMEOUT (kWaitCounter) in g_device_error and
// returns.
#pragma once

#include "fpemu_device.cuh"

namespace fpemu {

__device__ __forceinline__ void mc_store_16(void* mc_addr, uint4 v) {
    asm volatile("multimem.st.weak.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void mc_store_4(void* mc_addr, uint32_t v) {
    asm volatile("multimem.st.weak.global.b32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}

// counter += v on every GPU of the multicast group, ordered after this thread's
// earlier stores (and, through a preceding bar.sync, its CTA's).
__device__ __forceinline__ void mc_add_release(unsigned long long* mc_addr, unsigned long long v) {
    asm volatile("multimem.red.release.sys.global.add.u64 [%0], %1;" ::"l"(mc_addr), "l"(v) : "memory");
}

__device__ __forceinline__ void add_release(unsigned long long* addr, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long load_acquire(const unsigned long long* addr) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

constexpr int kMaxWaitCounters = 16;

struct CounterList {
    const unsigned long long* p[kMaxWaitCounters];  // local or peer-mapped counters
    int n;
};

// One thread waits until every listed counter is >= target.
__global__ void wait_counters_kernel(const __grid_constant__ CounterList L, unsigned long long target,
                                     int64_t budget_ns, int where) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const uint64_t t0 = global_ns();
    for (int i = 0; i < L.n; ++i) {
        while (load_acquire(L.p[i]) < target) {
            if ((int64_t)(global_ns() - t0) > budget_ns) {
                report_error(&g_device_error, FPEMU_ERR_TIMEOUT, kWaitCounter, where * kMaxWaitCounters + i);
                return;
            }
            __nanosleep(256);
        }
    }
}

// counter += 1 (multicast: on every GPU of the group) after everything earlier
// in the stream.
__global__ void signal_counter_kernel(unsigned long long* counter, int multicast) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    if (multicast) mc_add_release(counter, 1ull);
    else add_release(counter, 1ull);
}

}  // namespace fpemu
