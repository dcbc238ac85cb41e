// Streaming dequant-GEMV engine shared by the decode kernels.
//
// Work is cut into units of 16 weight rows x full K.  A producer warp moves
// each unit's raw GGUF rows from HBM into a ring of shared-memory stages
// with 1-D bulk copies (TMA engine, mbarrier completion); W consumer warps
// split each unit's K into 256-value segments, round-robin over the whole
// (unit, segment) sequence, and run the tensor-core segment kernels below.
// Each warp leaves one 16-row partial per unit in shared memory; the last
// warp to finish a unit sums the W partials in warp order (deterministic)
// and runs the caller's epilogue.
//
// Stage layout: rows 0..7 ("half 0") and 8..15 ("half 1") may come from
// different matrices (gate and up rows of one expert).  Rows are copied
// one by one when a row is a multiple of 16 bytes (padded so consecutive
// rows start 16 B apart modulo 128 B, which spreads the lanes of a warp over
// all 32 banks), or in dense groups of G rows when only G rows together
// form a multiple of 16 bytes.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "quant_frag.cuh"
#include "vireo_ptx.cuh"

namespace vireo {

constexpr int kMaxStages = 16;

struct StageGeom {
  uint32_t rb;       // bytes per weight row
  uint32_t G;        // rows per bulk copy (1, 2, 4 or 8)
  uint32_t gstride;  // smem bytes between copy groups inside a half
  uint32_t hstride;  // smem bytes from half 0 to half 1
};

VDEV const uint8_t* stage_row(const uint8_t* stage, const StageGeom& sg, int r) {
  int h = r >> 3, r8 = r & 7;
  return stage + h * sg.hstride + (r8 / (int)sg.G) * sg.gstride + (r8 % (int)sg.G) * sg.rb;
}

// Producer side: one thread issues the copies of a unit into a stage.
VDEV void issue_unit(uint8_t* stage, uint64_t* full, const uint8_t* src0, const uint8_t* src1,
                     const StageGeom& sg) {
  mbar_arrive_expect_tx(full, 16u * sg.rb);
  const uint32_t groups = 8u / sg.G, gbytes = sg.G * sg.rb;
  for (uint32_t j = 0; j < groups; j++) bulk_g2s(stage + j * sg.gstride, src0 + j * gbytes, gbytes, full);
  for (uint32_t j = 0; j < groups; j++)
    bulk_g2s(stage + sg.hstride + j * sg.gstride, src1 + j * gbytes, gbytes, full);
}

struct LaneCtx {
  int lane, g, t;
  uint32_t boff;
  bool bon;
};
VDEV LaneCtx lane_ctx() {
  LaneCtx c;
  c.lane = threadIdx.x & 31;
  c.g = c.lane >> 2;
  c.t = c.lane & 3;
  c.boff = (uint32_t)(c.t * 16 + (c.g & 1) * 8);
  c.bon = ((c.g >> 1) == c.t);
  return c;
}

VDEV void bload(const uint8_t* btab, int step, const LaneCtx& L, uint32_t& b0, uint32_t& b1) {
  uint2 v = lds64(btab + step * kStepBytesB + L.boff);
  b0 = L.bon ? v.x : 0u;
  b1 = L.bon ? v.y : 0u;
}

VDEV float h_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))); }
VDEV float h_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
VDEV uint32_t h2_splat(float v) {
  __half h = __float2half_rn(v);
  uint32_t u = (uint32_t)__half_as_ushort(h);
  return u | (u << 16);
}

// 16 bytes from a 2-byte-aligned shared address, as four words.
VDEV void ld16u(const uint8_t* p, uint32_t (&w)[4]) {
  uint32_t a = smem_addr(p);
  uint32_t a4 = a & ~3u, sh = (a & 2u) << 3;
  uint32_t x0, x1, x2, x3, x4;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x0) : "r"(a4));
  asm volatile("ld.shared.u32 %0, [%1+4];" : "=r"(x1) : "r"(a4));
  asm volatile("ld.shared.u32 %0, [%1+8];" : "=r"(x2) : "r"(a4));
  asm volatile("ld.shared.u32 %0, [%1+12];" : "=r"(x3) : "r"(a4));
  asm volatile("ld.shared.u32 %0, [%1+16];" : "=r"(x4) : "r"(a4));
  w[0] = __funnelshift_r(x0, x1, sh);
  w[1] = __funnelshift_r(x1, x2, sh);
  w[2] = __funnelshift_r(x2, x3, sh);
  w[3] = __funnelshift_r(x3, x4, sh);
}
VDEV int lds_s8(const void* p) {
  int v;
  asm volatile("ld.shared.s8 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)));
  return v;
}
VDEV uint32_t lds_u16(const void* p) {
  uint32_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)));
  return v;
}

// ---------------------------------------------------------------------------
// Segment kernels: accumulate one 256-value segment of rows g (r0) and g+8
// (r1) into this lane's fp32 totals.  btab: the segment's B table
// (16 steps x 64 B); sx: the segment's 8 sub-block sums (Q4_K only).
// ---------------------------------------------------------------------------
struct SegQ8 : Q8 {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const uint8_t* btab, const float* sx,
                       const LaneCtx& L, float& tot0, float& tot1) {
    (void)sx;
    const uint8_t* p0 = r0 + 68 * L.t;
    const uint8_t* p1 = r1 + 68 * L.t;
    const uint32_t w0a = lds32(p0), w8a = lds32(p0 + 32), w0b = lds32(p1), w8b = lds32(p1 + 32);
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 8; s++) {
      uint32_t wa = (s < 7) ? lds32(p0 + 4 + 4 * s) : byte_perm(w0a, w8a, 0x5432u);
      uint32_t wb = (s < 7) ? lds32(p1 + 4 + 4 * s) : byte_perm(w0b, w8b, 0x5432u);
      uint32_t a[4];
      conv(wa, a[0], a[2]);
      conv(wb, a[1], a[3]);
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = h2_sub(a[i], kBias);
      uint32_t b0, b1;
      bload(btab, s, L, b0, b1);
      mma_16816(c, a, b0, b1);
    }
    tot0 += h_lo(w0a) * (c[0] + c[1]);
    tot1 += h_lo(w0b) * (c[2] + c[3]);
    c[0] = c[1] = c[2] = c[3] = 0.f;
#pragma unroll
    for (int s = 0; s < 8; s++) {
      uint32_t wa = lds32(p0 + 36 + 4 * s), wb = lds32(p1 + 36 + 4 * s);
      uint32_t a[4];
      conv(wa, a[0], a[2]);
      conv(wb, a[1], a[3]);
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = h2_sub(a[i], kBias);
      uint32_t b0, b1;
      bload(btab, 8 + s, L, b0, b1);
      mma_16816(c, a, b0, b1);
    }
    tot0 += h_hi(w8a) * (c[0] + c[1]);
    tot1 += h_hi(w8b) * (c[2] + c[3]);
  }
};

struct SegQ4K : Q4K {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const uint8_t* btab, const float* sx,
                       const LaneCtx& L, float& tot0, float& tot1) {
    const uint4 hd0 = lds128(r0), hd1 = lds128(r1);
    const int j0 = 2 * L.t, j1 = 2 * L.t + 1;
    uint32_t sc00, mn00, sc01, mn01, sc10, mn10, sc11, mn11;
    scale_min(hd0.y, hd0.z, hd0.w, j0, sc00, mn00);
    scale_min(hd0.y, hd0.z, hd0.w, j1, sc01, mn01);
    scale_min(hd1.y, hd1.z, hd1.w, j0, sc10, mn10);
    scale_min(hd1.y, hd1.z, hd1.w, j1, sc11, mn11);
    // low nibbles (sub-block 2t): A = sc*(1024+q) - 1024*sc ; high nibbles
    // (sub-block 2t+1, stored as 1024+16q): A = (sc/16)*(1024+16q) - 64*sc
    const uint32_t SL0 = h2_splat((float)sc00), CL0 = h2_splat(-1024.f * (float)sc00);
    const uint32_t SH0 = h2_splat((float)sc01 * 0.0625f), CH0 = h2_splat(-64.f * (float)sc01);
    const uint32_t SL1 = h2_splat((float)sc10), CL1 = h2_splat(-1024.f * (float)sc10);
    const uint32_t SH1 = h2_splat((float)sc11 * 0.0625f), CH1 = h2_splat(-64.f * (float)sc11);
    const uint4 qa0 = lds128(r0 + 16 + 32 * L.t), qa1 = lds128(r0 + 32 + 32 * L.t);
    const uint4 qb0 = lds128(r1 + 16 + 32 * L.t), qb1 = lds128(r1 + 32 + 32 * L.t);
    const uint32_t wa[8] = {qa0.x, qa0.y, qa0.z, qa0.w, qa1.x, qa1.y, qa1.z, qa1.w};
    const uint32_t wb[8] = {qb0.x, qb0.y, qb0.z, qb0.w, qb1.x, qb1.y, qb1.z, qb1.w};
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      uint32_t a[4], t02, t13, b0, b1;
      conv_lo(wa[i], t02, t13);
      a[0] = h2_fma(t02, SL0, CL0);
      a[2] = h2_fma(t13, SL0, CL0);
      conv_lo(wb[i], t02, t13);
      a[1] = h2_fma(t02, SL1, CL1);
      a[3] = h2_fma(t13, SL1, CL1);
      bload(btab, 2 * i, L, b0, b1);
      mma_16816(c, a, b0, b1);
      conv_hi(wa[i], t02, t13);
      a[0] = h2_fma(t02, SH0, CH0);
      a[2] = h2_fma(t13, SH0, CH0);
      conv_hi(wb[i], t02, t13);
      a[1] = h2_fma(t02, SH1, CH1);
      a[3] = h2_fma(t13, SH1, CH1);
      bload(btab, 2 * i + 1, L, b0, b1);
      mma_16816(c, a, b0, b1);
    }
    const float sxa = sx[j0], sxb = sx[j1];
    const float mt0 = (float)mn00 * sxa + (float)mn01 * sxb;
    const float mt1 = (float)mn10 * sxa + (float)mn11 * sxb;
    tot0 += h_lo(hd0.x) * (c[0] + c[1]) - h_hi(hd0.x) * mt0;
    tot1 += h_lo(hd1.x) * (c[2] + c[3]) - h_hi(hd1.x) * mt1;
  }
};

struct SegQ6K : Q6K {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const uint8_t* btab, const float* sx,
                       const LaneCtx& L, float& tot0, float& tot1) {
    (void)sx;
    const float d0 = __half2float(__ushort_as_half((unsigned short)lds_u16(r0 + 208)));
    const float d1 = __half2float(__ushort_as_half((unsigned short)lds_u16(r1 + 208)));
    const int qlo = 32 * (L.t & 1);
#pragma unroll
    for (int m = 0; m < 4; m++) {
      const int h = m >> 1, l0 = 16 * (m & 1);
      uint32_t la[4], ha[4], lb[4], hb[4];
      ld16u(r0 + 64 * h + qlo + l0, la);
      ld16u(r0 + 128 + 32 * h + l0, ha);
      ld16u(r1 + 64 * h + qlo + l0, lb);
      ld16u(r1 + 128 + 32 * h + l0, hb);
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 4; s++) {
        uint32_t a[4], b0, b1;
        conv(six(la[s], ha[s], L.t), a[0], a[2]);
        conv(six(lb[s], hb[s], L.t), a[1], a[3]);
#pragma unroll
        for (int i = 0; i < 4; i++) a[i] = h2_sub(a[i], kBias);
        bload(btab, 4 * m + s, L, b0, b1);
        mma_16816(c, a, b0, b1);
      }
      const int sidx = 192 + 8 * h + 2 * L.t + (m & 1);
      const float s0 = (float)lds_s8(r0 + sidx), s1 = (float)lds_s8(r1 + sidx);
      tot0 += (d0 * s0) * (c[0] + c[1]);
      tot1 += (d1 * s1) * (c[2] + c[3]);
    }
  }
};

// ---------------------------------------------------------------------------
// B tables: an fp32 vector v[K] scaled by a power of two (so that max|v|
// lands in [2^14, 2^15) and the f16 split neither overflows nor flushes),
// split into x_hi + x_lo and laid out in each format's k order.
// ---------------------------------------------------------------------------

// power-of-two scale for a vector whose max magnitude is amax
VDEV float pow2_scale(float amax) {
  if (!(amax > 0.f) || !isfinite(amax)) return 1.f;
  int ex;
  frexpf(amax, &ex);  // amax in [2^(ex-1), 2^ex)
  int e = 15 - ex;
  e = e > 100 ? 100 : (e < -100 ? -100 : e);
  return ldexpf(1.f, e);
}

// Block-cooperative (threads tid in [0, nthr)).  v may be global or shared.
template <class F>
VDEV void build_btab(const float* v, int K, float scale, uint8_t* tab, float* sx, int tid, int nthr,
                     bool from_global) {
  for (int idx = tid; idx < K; idx += nthr) {
    const int seg = idx >> 8, rem = idx & 255;
    const int step = rem >> 4, t = (rem >> 2) & 3, j = rem & 3;
    const int e = seg * kSegElems + F::elem(step, t, j);
    const float x = (from_global ? __ldcg(v + e) : v[e]) * scale;
    const __half hi = __float2half_rn(x);
    const __half lo = __float2half_rn(x - __half2float(hi));
    uint8_t* dst = tab + seg * (16 * kStepBytesB) + step * kStepBytesB + t * 16 + j * 2;
    *reinterpret_cast<__half*>(dst) = hi;
    *reinterpret_cast<__half*>(dst + 8) = lo;
  }
  if (F::kNeedsSubSums) {
    for (int i = tid; i < K / 32; i += nthr) {
      float s = 0.f;
      for (int l = 0; l < 32; l++) s += (from_global ? __ldcg(v + 32 * i + l) : v[32 * i + l]) * scale;
      sx[i] = s;
    }
  }
}

// ---------------------------------------------------------------------------
// Consumer side of one unit for warp w: run this warp's segments, reduce
// over the 4 lanes of a row, publish the 16-row partial, and return true in
// the warp that completes the unit (which then owns the epilogue with the
// summed rows in lanes 0..15 via *row_val).
// ---------------------------------------------------------------------------
template <class S>
VDEV bool consume_unit(const uint8_t* stage, const StageGeom& sg, int v, int nseg, int W, int w,
                       const uint8_t* btab, const float* sx, float* part /*[W][16]*/, int* ucnt,
                       const LaneCtx& L, float* row_val) {
  const uint8_t* r0 = stage_row(stage, sg, L.g);
  const uint8_t* r1 = stage_row(stage, sg, L.g + 8);
  float tot0 = 0.f, tot1 = 0.f;
  int first = (w - (v * nseg) % W) % W;
  if (first < 0) first += W;
  for (int seg = first; seg < nseg; seg += W)
    S::run(r0 + seg * S::kSegBytes, r1 + seg * S::kSegBytes, btab + seg * (16 * kStepBytesB), sx + seg * 8,
           L, tot0, tot1);
  tot0 += __shfl_xor_sync(0xffffffffu, tot0, 1);
  tot1 += __shfl_xor_sync(0xffffffffu, tot1, 1);
  tot0 += __shfl_xor_sync(0xffffffffu, tot0, 2);
  tot1 += __shfl_xor_sync(0xffffffffu, tot1, 2);
  if (L.t == 0) {
    part[w * 16 + L.g] = tot0;
    part[w * 16 + L.g + 8] = tot1;
  }
  __syncwarp();
  int last = 0;
  if (L.lane == 0) {
    __threadfence_block();
    last = (atomicAdd(ucnt, 1) == W - 1);
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence_block();
    float acc = 0.f;
    if (L.lane < 16)
      for (int ww = 0; ww < W; ww++) acc += ((volatile float*)part)[ww * 16 + L.lane];
    *row_val = acc;
    __syncwarp();
    if (L.lane == 0) *ucnt = 0;
  }
  return last != 0;
}

}  // namespace vireo
