// Fifth-generation tensor cores (tcgen05) and tiled TMA on sm_100a: thin
// PTX wrappers used by the prefill GEMMs.
//
// Operand layout used throughout: K-major tiles in shared memory with the
// 128-byte swizzle, one row = 64 f16 (128 B) of K, 8-row groups 1024 B
// apart, tile base 1024-byte aligned.  That is the layout a 2-D TMA load
// with CU_TENSOR_MAP_SWIZZLE_128B and a box of {64, rows} writes, and the
// one a thread writing row r's 16-byte chunk c at r * 128 + ((c ^ (r & 7))
// * 16) produces.  The UMMA shared-memory descriptor of such a tile: start
// address >> 4 (bits 0-13), leading byte offset 1 (unused with swizzle, bits
// 16-29), stride byte offset 1024 >> 4 (bits 32-45), descriptor version 1
// (bit 46), layout SWIZZLE_128B = 2 (bits 61-63); the k-th 16-wide K slice
// of the tile starts 32 * k bytes further (start field + 2 k).
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "vireo_ptx.cuh"

namespace vireo {

VDEV uint64_t umma_desc_sw128(const void* tile) {
  const uint64_t a = (smem_addr(tile) >> 4) & 0x3FFFu;
  return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// instruction descriptor of kind::f16: A, B f16 (both K-major), D f32,
// M x N; bits: D format 4-5 (1 = f32), A/B format 7-9/10-12 (0 = f16),
// A/B major 15/16 (0 = K), N >> 3 at 17-22, M >> 4 at 24-28
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread
VDEV void umma_f16_ss(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}
// arrive (once) on bar when every tcgen05.mma this thread issued so far is done
VDEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
VDEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
VDEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMEM allocation: one whole warp; the column base is written to *slot
VDEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
VDEV void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

// 32 consecutive 32-bit columns of the calling warp's 32 TMEM lanes (warp w
// of a warpgroup reads lanes 32 (w % 4) ..): thread = lane, v[j] = column j
VDEV void tmem_ld32(uint32_t addr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2-D tiled TMA load (one CTA, this GPU's memory) completing on bar; x (innermost, in
// elements) must be a multiple of 16 bytes' worth of elements
VDEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
// make this thread's generic-proxy shared-memory writes visible to the
// async proxy (the tensor core reading the tile)
VDEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace vireo
