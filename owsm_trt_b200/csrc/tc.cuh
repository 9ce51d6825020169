// Fifth-generation tensor-core (tcgen05) and tensor-copy (TMA) building blocks for sm_100a, as inline PTX.
//
// * TMEM: a CTA allocates accumulator columns (a power of two >= 32 of the 512 x 32-bit columns of its SM) with
//   one warp, and frees them with the same warp before it exits. An address is (lane << 16) | column; warp w of
//   a CTA reads lanes 32 (w % 4) .. 32 (w % 4) + 31.
// * MMA: one thread issues tcgen05.mma.cta_group::1.kind::f16 (fp16 A and B from shared memory, fp32
//   accumulator in TMEM), D[M x N] (+)= A[M x 16] B[N x 16]^T; the operands are described by 64-bit shared-memory
//   descriptors, the shape and types by a 32-bit instruction descriptor. tcgen05.commit makes an mbarrier
//   arrive once every MMA the thread issued before it has completed (operands read, accumulator written).
// * TMA: cp.async.bulk.tensor.2d loads a box of a row-major tensor (described by a CUtensorMap in kernel
//   parameter space) into shared memory with the 128-byte swizzle the descriptors below expect; completion is
//   counted in bytes on an mbarrier. No multicast.
//
// Descriptor fields follow the PTX ISA's tcgen05 "shared memory descriptor" and "instruction descriptor"
// tables (the bit positions CUTLASS's cute/arch/mma_sm100_desc.hpp also uses).
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace owsm {

// ---------------------------------------------------------------- TMEM
// All 32 lanes of one warp execute these.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Order tcgen05 operations of this thread against a thread barrier / an mbarrier wait that follows (before) or
// precedes (after) them.
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------------------------------------------------------- MMA
// Shared-memory descriptor of a K-major operand tile stored with the 128-byte swizzle (rows of 64 fp16 = 128
// bytes, groups of 8 rows = 1024 bytes apart; the tile 1024-byte aligned): start address >> 4 in bits 0-13,
// leading byte offset (unused by swizzled K-major layouts; 16 bytes) in 16-29, stride byte offset 1024 >> 4 in
// 32-45, the descriptor version 1 in 46-47, base offset 0, layout 2 (128-byte swizzle) in 61-63. Successive
// K = 16 slices of a 64-wide swizzle row start 32 bytes further (the swizzle is a function of the address).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Shared-memory descriptor of a K-major operand without swizzle ("interleaved" core matrices of 8 rows x 16
// bytes, 128 contiguous bytes each): lbo = bytes between core matrices adjacent in K, sbo = bytes between core
// matrices adjacent in M / N.
__device__ __forceinline__ uint64_t plain_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// Instruction descriptor, kind::f16 with fp16 A and B (both K-major), fp32 accumulator: D format 1 (F32) in
// bits 4-5, A / B format 0 (F16) in 7-9 / 10-12, N >> 3 in 17-22, M >> 4 in 24-28.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D (tmem) = A B^T (+ D when accumulate != 0); one thread.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// `bar` (this CTA's shared memory) receives one arrival when every tcgen05.mma this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane (warp-wide; lane quarter fixed by the warp).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- TMA
// Box (x = inner coordinate, y = row) of the tensor `map` (address of a __grid_constant__ kernel parameter)
// into shared memory at dst; bytes counted on bar. x * element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Contiguous bytes global -> this CTA's shared memory by the bulk-copy engine, counted on bar (no cache hint).
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s_nohint(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Make this thread's ordinary shared-memory writes visible to the async proxy (tensor-core operand reads).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace owsm
