#pragma once

// Inline-PTX wrappers for sm_100a: mbarriers with bounded waits, TMA tile
// loads (no multicast), tcgen05 MMA / commit / fences / TMEM loads, and the
// shared-memory and instruction descriptors for K-major int8 tiles with a
// 128-byte swizzle.

#include <cuda.h>
#include <cstdint>

namespace nvcr_sm100::kernels {

constexpr int tile_positions_m = 128;  // MMA M: output positions per tile
constexpr int tile_k_bytes = 128;      // K bytes per stage: one 128-byte swizzle row
constexpr unsigned long long wait_limit_ns = 2000000000ull;

static __device__ __forceinline__ std::uint32_t smem_address(const void* p) {
    return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

static __device__ __forceinline__ unsigned long long global_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

static __device__ __forceinline__ void barrier_init(std::uint32_t bar, std::uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

static __device__ __forceinline__ void barrier_expect_bytes(std::uint32_t bar, std::uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

static __device__ __forceinline__ bool barrier_try_wait(std::uint32_t bar, std::uint32_t parity) {
    std::uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Non-blocking: whether the phase of `parity` has completed.
static __device__ __forceinline__ bool barrier_test_wait(std::uint32_t bar, std::uint32_t parity) {
    std::uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase of `parity` to complete; false (and status bit 0) once
// `limit_ns` of the global timer have passed.
static __device__ bool barrier_wait_for(std::uint32_t bar, std::uint32_t parity, unsigned int* status,
                                        unsigned long long limit_ns) {
    if (barrier_try_wait(bar, parity)) return true;
    const unsigned long long start = global_timer();
    for (unsigned int spin = 0;; ++spin) {
        if (barrier_try_wait(bar, parity)) return true;
        if ((spin & 63u) == 63u) {
            if (global_timer() - start > limit_ns) {
                atomicOr(status, 1u);
                return false;
            }
            __nanosleep(128);
        }
    }
}

// The same with the kernels' limit of about two seconds.
static __device__ bool barrier_wait(std::uint32_t bar, std::uint32_t parity, unsigned int* status) {
    return barrier_wait_for(bar, parity, status, wait_limit_ns);
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about `hint_ns` have passed, issuing nothing meanwhile.
static __device__ __forceinline__ bool barrier_try_wait_hint(std::uint32_t bar, std::uint32_t parity,
                                                             std::uint32_t hint_ns) {
    std::uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return done != 0;
}

// barrier_wait for warps that share a sub-partition with a latency-critical
// thread: the waiting thread is suspended in hardware (woken when the phase
// completes) instead of polling, so it takes no issue slots; the same limit of
// about two seconds, after which status bit 0 is set and false returned.
static __device__ bool barrier_sleep_wait(std::uint32_t bar, std::uint32_t parity, unsigned int* status) {
    if (barrier_try_wait_hint(bar, parity, 50000u)) return true;
    const unsigned long long start = global_timer();
    for (;;) {
        if (barrier_try_wait_hint(bar, parity, 50000u)) return true;
        if (global_timer() - start > wait_limit_ns) {
            atomicOr(status, 1u);
            return false;
        }
    }
}

static __device__ __forceinline__ void tma_load_2d(std::uint32_t dst, const CUtensorMap* map, std::uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<std::uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

static __device__ __forceinline__ void tma_load_3d(std::uint32_t dst, const CUtensorMap* map, std::uint32_t bar, int x,
                                                   int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<std::uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major tile with 128-byte swizzle:
// 8-row x 128-byte atoms stacked 1024 bytes apart (SBO), LBO unused (1),
// descriptor version 1 (bits 46-47), layout 2 = SWIZZLE_128B (bits 61-63).
static __device__ __forceinline__ std::uint64_t sw128_descriptor(std::uint32_t address) {
    return static_cast<std::uint64_t>((address >> 4) & 0x3FFFu) | (static_cast<std::uint64_t>(1) << 16) |
        (static_cast<std::uint64_t>(1024 >> 4) << 32) | (static_cast<std::uint64_t>(1) << 46) |
        (static_cast<std::uint64_t>(2) << 61);
}

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A and B signed 8-bit
// (bits 7-9 and 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
static __device__ __forceinline__ std::uint32_t i8_instruction(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<std::uint32_t>(n >> 3) << 17) |
        (static_cast<std::uint32_t>(tile_positions_m >> 4) << 24);
}

static __device__ __forceinline__ void mma_i8(std::uint32_t d_tmem, std::uint64_t a, std::uint64_t b, std::uint32_t idesc,
                                       std::uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

static __device__ __forceinline__ void mma_commit(std::uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

static __device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
static __device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this thread's lane.
static __device__ __forceinline__ void tmem_load16(std::uint32_t address, int (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(address));
}

static __device__ __forceinline__ void tmem_load_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 TMEM lanes x 16 32-bit columns in the mma accumulator fragment layout:
// thread t holds (lane t/4, columns 2(t%4), 2(t%4)+1) in r0, r1 and lane
// t/4 + 8 of the same columns in r2, r3; r4..r7 the same for columns 8..15.
static __device__ __forceinline__ void tmem_load_16x256b_x2(std::uint32_t address, std::uint32_t* r) {
    asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(address));
}

// tcgen05.wait::ld that also carries the loaded registers, so no use of them
// can be scheduled before the wait.
static __device__ __forceinline__ void tmem_load_wait_regs(std::uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// Four 8x8 matrices of 16-bit elements, each stored transposed: lane l gives
// the shared address of row l % 8 of matrix l / 8, which receives column l % 8
// of that matrix from the fragment (thread t holding elements 2(t%4), 2(t%4)+1
// of row t/4 in register i for matrix i).
static __device__ __forceinline__ void stmatrix_x4_trans(std::uint32_t address, const std::uint32_t (&r)[4]) {
    asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(address), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3])
                 : "memory");
}

static __device__ __forceinline__ uint4 load_shared_v4(std::uint32_t address) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(address)
                 : "memory");
    return v;
}

// Arrive (count one) on an mbarrier from a generic-proxy thread.
static __device__ __forceinline__ void barrier_arrive(std::uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the
// async proxy (the tensor cores read operands through it).
static __device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace nvcr_sm100::kernels
