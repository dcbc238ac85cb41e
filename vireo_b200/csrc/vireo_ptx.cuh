// Thin wrappers over the sm_100a PTX this library uses: mbarriers, 1-D bulk
// async copies (TMA engine, global -> shared), warp-level f16 tensor-core
// MMA, f16x2 arithmetic, and bounded waits.  Every wait in this library is
// bounded by a wall-clock limit read from %globaltimer; a wait that runs out
// records VIREO_ERR_TIMEOUT in a device status word and returns false so
// the kernel can drain its copies and exit instead of hanging the GPU.
#pragma once
#include <cuda_fp16.h>
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
// try_wait that lets the hardware suspend the thread for up to hint_ns
VDEV bool mbar_test_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Suspend-time hint of the barrier waits, in ns (0: the hardware's default).
#ifndef VIREO_MBAR_HINT_NS
#define VIREO_MBAR_HINT_NS 0
#endif

// Waits for the phase with the given parity to complete: try_wait in a loop
// (each try may suspend the thread, for at most the hint, and resumes it when
// the phase completes).  Gives up (false) when the time limit passes or
// *abort becomes non-zero.
VDEV bool mbar_wait(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  if (mbar_test(bar, parity)) return true;
  uint64_t t0 = now_ns();
  for (;;) {
    if (VIREO_MBAR_HINT_NS ? mbar_test_suspend(bar, parity, VIREO_MBAR_HINT_NS) : mbar_test(bar, parity)) return true;
    if (*abort) return false;
    if (now_ns() - t0 > kWaitLimitNs) return false;
  }
}
// warp-collective wait: lane 0 waits, the warp then proceeds together (the
// __syncwarp orders the other lanes' later shared-memory reads after the
// completed phase).  Returns the same result in every lane.
VDEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
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

// ---- 16-byte asynchronous copies global -> shared (LSU path) --------------
VDEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
// arrive on bar once every cp.async this thread issued so far has landed
// (the barrier's expected count includes this arrival)
VDEV void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
VDEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---- programmatic dependent launch ---------------------------------------
// wait until the preceding kernel in the stream has completed and its
// memory is visible (no-op when launched without the PDL attribute)
VDEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// allow the next kernel in the stream to begin launching
VDEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- tensor core: D = A(16x16 f16) * B(16x8 f16) + C, fp32 accumulate ----
VDEV void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- shared-memory matrix loads for the f16 MMA operands -----------------
// Four 8x8 b16 matrices: lane l supplies the address of row l % 8 of matrix
// l / 8 (16 bytes, 16-byte aligned); register i receives matrix i in the MMA
// fragment layout (lane 4 g + t: row g, columns 2t, 2t + 1), or, with
// .trans, the transposed matrix.
VDEV void ldsm_x4(const void* row, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_addr(row))
               : "memory");
}
VDEV void ldsm_x4_trans(const void* row, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_addr(row))
               : "memory");
}
// two floats as one f16x2 register (lo = a), round to nearest
VDEV uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// ---- integer tensor core: D = A(16x32 int8) * B(32x8 s8) (+ C), s32 ------
// Fragments (lane = 4 g + t): A regs {row g, k 4t..4t+3}, {row g+8, same k},
// {row g, k 16+4t..}, {row g+8, k 16+4t..}; B regs {k 4t..4t+3, col g},
// {k 16+4t.., col g}; C {row g: cols 2t, 2t+1}, {row g+8: cols 2t, 2t+1}.
// The first MMA of a chain starts from zero (imma_*_z), the rest accumulate.
VDEV void imma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
VDEV void imma_s8_z(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}
VDEV void imma_u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
VDEV void imma_u8_z(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
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
// Plain C++ loads (not asm volatile) so the compiler may schedule them ahead
// of their use; they stay ordered after the mbarrier waits, which clobber
// memory.  Pointers are derived from the kernel's shared arrays, so these
// compile to shared-memory loads.
VDEV uint32_t lds32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }
VDEV uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }
VDEV uint2 lds64(const void* p) { return *reinterpret_cast<const uint2*>(p); }

// ---- global loads that bypass L1 (data written by other CTAs) ------------
VDEV uint32_t ld_acquire_gpu(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

VDEV void st_release_gpu(unsigned int* p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
VDEV unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
VDEV void red_add_release_gpu(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// L2 prefetch of a 16-byte-aligned span (size a multiple of 16)
VDEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Waits until *p >= target (acquire).  One thread per CTA polls.  Returns
// false on timeout (recorded in *err) or when *err is already set.
VDEV bool wait_geq(unsigned int* p, unsigned int target, int* err) {
  if (ld_acquire_gpu(p) >= target) return true;
  uint64_t t0 = now_ns();
  for (;;) {
    __nanosleep(32);
    if (ld_acquire_gpu(p) >= target) return true;
    if (*(volatile int*)err) return false;
    if (now_ns() - t0 > kWaitLimitNs) {
      atomicCAS(err, 0, VIREO_ERR_TIMEOUT);
      return false;
    }
  }
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
