// tc.cuh -- building blocks of the tensor-core kernels (tcgen05, mbarriers,
// bulk and tensor copies), shared by route_tc.cu and exact_tc.cu.
//
// Every wait here is bounded (kTCWaitNs of wall time, read from the global
// timer; the polls suspend the waiting thread in between, so that waiting
// warps do not take issue slots): a kernel whose wait gives up reports it
// through its error flag instead of hanging the device.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace isb {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// byte offset of the 16-byte chunk (row, k8) -- elements k = 8*k8 .. 8*k8+7 --
// in the canonical layout of an operand of R rows
__host__ __device__ __forceinline__ size_t tc_chunk_off(int row, int k8, int R) {
    return (size_t)(k8 >> 1) * ((size_t)R * 32) + (size_t)(row >> 3) * 256 + (size_t)(k8 & 1) * 128 +
           (size_t)(row & 7) * 16;
}

// shared-memory matrix descriptor, K-major without swizzle: 8-row x 16-byte
// core matrices, the two halves of one MMA's 32 bytes of K 128 bytes apart
// (leading byte offset), 8-row groups 256 bytes apart (stride byte offset)
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);          // start address, 16-byte units
    d |= (uint64_t)(128u >> 4) << 16;                  // leading byte offset: K halves
    d |= (uint64_t)(256u >> 4) << 32;                  // stride byte offset: 8-row groups
    d |= (uint64_t)1 << 46;                            // descriptor version of sm_100
    return d;                                          // base offset 0, no swizzle
}

// shared-memory matrix descriptor, K-major with the 128-byte swizzle: rows of
// 128 bytes, the 16-byte chunk c of row r stored at chunk c ^ (r % 8), 8-row
// atoms of 1024 bytes one after another (stride byte offset).  The atom base
// must be 1024-byte aligned; the start address may step through the 128 bytes
// of K (32 bytes per MMA of 8-bit operands).  The leading byte offset is not
// used by this layout.
__device__ __forceinline__ uint64_t umma_smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);          // start address, 16-byte units
    d |= (uint64_t)1 << 16;                            // leading byte offset (unused)
    d |= (uint64_t)(1024u >> 4) << 32;                 // stride byte offset: 8-row atoms
    d |= (uint64_t)1 << 46;                            // descriptor version of sm_100
    d |= (uint64_t)2 << 61;                            // layout: 128-byte swizzle
    return d;
}

// kind::f16 instruction descriptor: bf16 A and B (K-major), fp32 D, M x N
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// kind::i8 instruction descriptor: unsigned 8-bit A and B (K-major), s32 D
// (exact: at most 256 products of 255 x 255 per element), M x N
__host__ __device__ constexpr uint32_t umma_idesc_u8(int M, int N) {
    return (2u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// one try_wait that may suspend the thread (until the phase completes or
// about hint_ns pass), so that a waiting warp does not take issue slots
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

constexpr uint64_t kTCWaitNs = 2000000000ull;   // a wait gives up after 2 s

// wait on an mbarrier phase with suspending polls, bounded by kTCWaitNs of
// wall time; gives up early once *fail is set (fail may be null)
__device__ __forceinline__ bool mbar_wait_timed(uint64_t* bar, uint32_t parity, const volatile int* fail) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (fail && *fail) return false;
        if (globaltimer_ns() - t0 > kTCWaitNs) return false;
    }
}

// untiled bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// tiled tensor copy of the box at (x, y) of a 2-D tensor map into shared
// memory (no cluster multicast); x * element size must be a multiple of 16
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// the arrival on bar once every tcgen05 operation this thread issued so far is done
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes (one lane per thread)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace isb
