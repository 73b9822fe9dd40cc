// tc.cuh -- the 5th-generation tensor core (tcgen05) on sm_100a: tensor
// memory (TMEM) allocation, shared-memory matrix descriptors, the int8 MMA,
// its completion barrier and the TMEM loads of the epilogue, as inline PTX.
//
// Operands live in shared memory in the canonical K-major layout without
// swizzle: 8-row x 16-byte "core matrices" (128 contiguous bytes, row r of
// the core at byte 16 r); for a tile of R rows x 32 bytes (one K = 32 int8
// step) the core at (row group g, K chunk c) sits at byte 256 g + 128 c.  In
// descriptor terms the K-direction stride (LBO) is 128 bytes and the
// row-group stride (SBO) 256 bytes.
#pragma once
#include "common.cuh"

namespace qma {

// Byte offset of element (row, k) of a canonical K-major tile, 0 <= k < 32.
__host__ __device__ inline uint32_t tc_off(int row, int k) {
    return uint32_t((row >> 3) * 256 + (k >> 4) * 128 + (row & 7) * 16 + (k & 15));
}
constexpr uint32_t TC_LBO = 128, TC_SBO = 256;

// Shared-memory matrix descriptor (sm_100 layout): start address >> 4 in
// bits 0-13, leading-dimension byte offset >> 4 in bits 16-29, stride
// byte offset >> 4 in bits 32-45, descriptor version 1 in bits 46-47, base
// offset 0, no swizzle (layout type 0 in bits 61-63).
__device__ __forceinline__ uint64_t tc_desc(const void *smem_tile) {
    const uint32_t a = smem_addr(smem_tile);
    return uint64_t((a >> 4) & 0x3FFFu) | (uint64_t((TC_LBO >> 4) & 0x3FFFu) << 16) |
           (uint64_t((TC_SBO >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}

// Instruction descriptor of kind::i8: s8 x s8 -> s32, both K-major, M x N.
//   bits 4-5 accumulator format (2 = s32), 7-9 A format (1 = signed),
//   10-12 B format (1 = signed), 15 / 16 A / B major (0 = K),
//   17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t tc_idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// TMEM allocation by one full warp: ncols (a power of two >= 32) columns of
// 128 lanes x 32 bits; the address lands in *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, issued by one thread.
__device__ __forceinline__ void tc_mma_s8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          bool accumulate) {
    const uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(mask0), "r"(mask1), "r"(mask2),
        "r"(mask3)
        : "memory");
}
// The mbarrier receives one arrival when every MMA this thread issued
// before has completed (its results are in TMEM, its operands read).
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes visible to the tensor core's reads.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive TMEM columns of this warp's 32 lanes (lane quarter warp % 4):
// thread t gets row 32 (warp % 4) + t, columns col .. col + 31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// QMA_CUDA_MMA_SYNC=1 in the environment: the int8 GEMMs run on the previous
// tensor-core generation's warp-level MMAs (mma.sync) instead of tcgen05, as
// a cross-check (the same bits).
bool tc_disabled();
// Bounded waits of the dense tcgen05 GEMM that ran out (reset by reading).
int gemm_tc_wait_timeouts();

// mbarrier arrival by this thread (a plain count of arrivals)
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

}  // namespace qma
