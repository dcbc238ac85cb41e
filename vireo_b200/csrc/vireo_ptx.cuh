// Thin wrappers over the sm_100a PTX this library uses: mbarriers, 1-D bulk
// async copies (TMA engine, global -> shared), warp-level f16 tensor-core
// MMA, f16x2 arithmetic, and bounded waits.  Every wait in this library is
// bounded by a wall-clock limit read from %globaltimer; a wait that runs out
// records VIREO_ERR_TIMEOUT in a device status word and returns false so
// the kernel can drain its copies and exit instead of hanging the GPU.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "vireo_status.h"

#define VDEV __device__ __forceinline__

namespace vireo {

// 2 s: far above any legitimate wait in these kernels (microseconds).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

VDEV uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

VDEV uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ---- mbarrier -------------------------------------------------------------
VDEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
VDEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

VDEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
VDEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
VDEV bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete.  Gives up (false)
// when the time limit passes or *abort becomes non-zero.
VDEV bool mbar_wait(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  if (mbar_test(bar, parity)) return true;
  uint64_t t0 = now_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_test(bar, parity)) return true;
    if ((it & 63) == 63) {
      if (*abort) return false;
      if (now_ns() - t0 > kWaitLimitNs) return false;
    }
  }
}

// ---- 1-D bulk copy global -> shared (TMA engine), completes on mbarrier ---
// dst, src 16-byte aligned; bytes a multiple of 16.
VDEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---- tensor core: D = A(16x16 f16) * B(16x8 f16) + C, fp32 accumulate ----
VDEV void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- f16x2 on raw 32-bit registers (used only where results are exact) --
VDEV uint32_t h2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
VDEV uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ---- shared-memory loads --------------------------------------------------
VDEV uint32_t lds32(const void* p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)));
  return v;
}
VDEV uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_addr(p)));
  return v;
}
VDEV uint2 lds64(const void* p) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_addr(p)));
  return v;
}

// ---- global loads that bypass L1 (data written by other CTAs) ------------
VDEV uint32_t ld_acquire_gpu(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---- grid-wide barrier (one thread per CTA calls it) ---------------------
struct GridSync {
  unsigned int count;
  unsigned int gen;
};

// Returns false on timeout or when *err is already set.  Self-resetting:
// count returns to 0 at every completed barrier, so the state carries over
// between launches.
VDEV bool grid_barrier(GridSync* gs, unsigned int nblocks, int* err) {
  unsigned int g = ld_acquire_gpu(&gs->gen);
  __threadfence();
  unsigned int old = atomicAdd(&gs->count, 1u);
  if (old == nblocks - 1) {
    atomicExch(&gs->count, 0u);
    __threadfence();
    atomicAdd(&gs->gen, 1u);
    return true;
  }
  uint64_t t0 = now_ns();
  while (ld_acquire_gpu(&gs->gen) == g) {
    if (*(volatile int*)err) return false;
    if (now_ns() - t0 > kWaitLimitNs) {
      atomicCAS(err, 0, VIREO_ERR_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  __threadfence();
  return true;
}

VDEV void set_error(int* err, int code) { atomicCAS(err, 0, code); }

}  // namespace vireo
