// Asynchronous bulk copies (TMA engine) and mbarriers for sm_100a, with bounded waits.
//
// Every wait here gives up after a fixed number of polls, raises kErrTimeout in the caller's error word and returns
// false, so a logic error can never hang the GPU: the kernel finishes, the host reports the timeout.
#pragma once

#include "common.cuh"

namespace cb200 {

// About a second of polling at B200 clocks before a wait is declared stuck.
constexpr unsigned kMaxPolls = 1u << 26;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Ampere-style 16-byte asynchronous copies global -> shared, grouped by commit.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async proxy (TMA) before first use.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait for the phase with the given parity to complete. Returns false (and raises kErrTimeout) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned* err) {
    for (unsigned i = 0; i < kMaxPolls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicOr(err, kErrTimeout);
    return false;
}

// 1-D bulk copy global -> shared, completing `bytes` of transaction on `bar`. dst, src and bytes: multiples of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// ---- Cross-GPU flags (system scope) ---------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait of one thread until *flag >= epoch (flags never decrease; wrap-safe comparison), for flags another
// GPU raises. Gives up after `timeout_ns` of wall time (the global timer), raising kErrTimeout.
__device__ __forceinline__ bool wait_flag_geq(const unsigned* flag, unsigned epoch, unsigned long long timeout_ns,
                                             unsigned* err) {
    const unsigned long long start = global_ns();
    for (unsigned i = 0;; ++i) {
        if (int(ld_acquire_sys(flag) - epoch) >= 0) return true;
        if ((i & 63) == 63) {
            if (global_ns() - start > timeout_ns) break;
            __nanosleep(256);
        }
    }
    atomicOr(err, kErrTimeout);
    return false;
}

}  // namespace cb200
