// sm_100a tensor-core building blocks written as inline PTX: tensor memory
// (TMEM) allocation, tcgen05.mma (kind::f16, one CTA), its commit to an
// mbarrier, TMEM -> register loads, 2-D TMA tile loads and the shared-memory
// matrix descriptors of the UMMA canonical K-major SWIZZLE_128B layout.
//
// Layout used by every operand tile here: rows of 64 fp16 (128 bytes), eight
// rows form a 1024-byte swizzle atom, atoms are stacked at 1024-byte stride
// (SBO), and the 16-byte chunk c of row r sits at chunk c ^ (r & 7) -- the
// layout a TMA tile load with CU_TENSOR_MAP_SWIZZLE_128B produces.  Tiles
// start on 1024-byte boundaries.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include "common.cuh"

namespace inf {

// ---- TMEM ----------------------------------------------------------------
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
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 TMEM lanes x 8 consecutive 32-bit columns; thread t of the warp gets
// lane (lane_base + t).  taddr = base + (lane_base << 16) + column.
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- MMA -------------------------------------------------------------------
// D[tmem] (+)= A[smem] * B[smem]^T, fp16 operands, fp32 accumulate, M = 128.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrives (once) on `bar` when every tcgen05.mma this thread issued so far
// has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), A and
// B fp16 (bits 7-9, 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 at
// bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor, K-major SWIZZLE_128B: start address >> 4
// (bits 0-13), leading byte offset (unused by this layout; 1), stride byte
// offset 1024 >> 4 between 8-row atoms (bits 32-45), descriptor version 1
// (bits 46-47), layout SWIZZLE_128B = 2 (bits 61-63).  Advancing K by 16 fp16
// elements inside the 128-byte row adds 32 bytes (2 in the start field).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// byte offset of (row r, 16-byte chunk c) inside a SWIZZLE_128B tile
__device__ __forceinline__ uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// ---- TMA -------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 2-D tile (x = innermost element index, y = row) into shared memory,
// completion counted on `bar` in bytes.  x * element size must be a multiple
// of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace inf
