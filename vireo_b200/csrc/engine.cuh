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
  uint32_t G;        // rows per copy group (1, 2, 4 or 8)
  uint32_t gstride;  // smem bytes between copy groups inside a half
  uint32_t hstride;  // smem bytes from half 0 to half 1
  uint32_t gmagic;   // floor(b / (G * rb)) == (b * gmagic) >> 32 for b < 8 * rb
};

VDEV const uint8_t* stage_row(const uint8_t* stage, const StageGeom& sg, int r) {
  int h = r >> 3, r8 = r & 7;
  return stage + h * sg.hstride + (r8 / (int)sg.G) * sg.gstride + (r8 % (int)sg.G) * sg.rb;
}

// Producer side: nprod threads (ptid = 0..nprod-1) copy a unit into a stage
// in 16-byte pieces and each arrives on the stage's full barrier (expected
// count nprod) once its pieces have landed.  A null src0 issues nothing
// (the unit is skipped) but still arrives.
// Each half (8 rows, contiguous in global memory) is walked as one flat
// byte range so that consecutive lanes copy consecutive 16-byte pieces; the
// destination of a piece is its copy group's padded slot, found with a
// multiply-shift division.
VDEV void issue_unit(uint8_t* stage, uint64_t* full, const uint8_t* src0, const uint8_t* src1,
                     const StageGeom& sg, int ptid, int nprod) {
  if (src0) {
    const uint32_t gbytes = sg.G * sg.rb;  // bytes per copy group (multiple of 16)
    const uint32_t hbytes = 8u * sg.rb;
#pragma unroll
    for (uint32_t h = 0; h < 2; h++) {
      const uint8_t* hs = h ? src1 : src0;
      uint8_t* hd = stage + h * sg.hstride;
      for (uint32_t b = 16u * (uint32_t)ptid; b < hbytes; b += 16u * (uint32_t)nprod) {
        const uint32_t j = __umulhi(b, sg.gmagic);
        cp_async16(hd + j * sg.gstride + (b - j * gbytes), hs + b);
      }
    }
  }
  cp_async_arrive(full);
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
  uint32_t sh = (a & 2u) << 3;
  const uint32_t* q = reinterpret_cast<const uint32_t*>(p - (a & 3u));
  const uint32_t x0 = q[0], x1 = q[1], x2 = q[2], x3 = q[3], x4 = q[4];
  w[0] = __funnelshift_r(x0, x1, sh);
  w[1] = __funnelshift_r(x1, x2, sh);
  w[2] = __funnelshift_r(x2, x3, sh);
  w[3] = __funnelshift_r(x3, x4, sh);
}
VDEV int lds_s8(const void* p) { return *reinterpret_cast<const int8_t*>(p); }
VDEV uint32_t lds_u16(const void* p) { return *reinterpret_cast<const uint16_t*>(p); }

// ---------------------------------------------------------------------------
// B fragments of one segment held in registers (16 steps x 2 regs); a warp
// that meets the same segment of the same table again (consecutive units
// whose segment index lands on the same warp) skips the reload.
// ---------------------------------------------------------------------------
struct BFrag {
  uint32_t b[16][2];
  const uint8_t* key;
  VDEV void reset() { key = nullptr; }
  VDEV void get(const uint8_t* segtab, const LaneCtx& L) {
    if (segtab == key) return;
    key = segtab;
#pragma unroll
    for (int s = 0; s < 16; s++) {
      const uint2 v = lds64(segtab + s * kStepBytesB + L.boff);
      b[s][0] = L.bon ? v.x : 0u;
      b[s][1] = L.bon ? v.y : 0u;
    }
  }
};

// ---------------------------------------------------------------------------
// Segment kernels: accumulate one 256-value segment of rows g (r0) and g+8
// (r1) into this lane's fp32 totals.  B: the segment's fragments; sx: the
// segment's 8 sub-block sums (Q4_K only).  Each kernel runs two independent
// accumulator chains so consecutive tensor-core ops do not wait on each
// other.
// ---------------------------------------------------------------------------
struct SegQ8 : Q8 {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const BFrag& B, const float* sx, const LaneCtx& L,
                       float& tot0, float& tot1) {
    const uint8_t* p0 = r0 + 68 * L.t;
    const uint8_t* p1 = r1 + 68 * L.t;
    const uint32_t w0a = lds32(p0), w8a = lds32(p0 + 32), w0b = lds32(p1), w8b = lds32(p1 + 32);
    float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 8; s++) {
      // block A (steps 0..7) and block B (steps 8..15) interleaved
      const uint32_t wa = (s < 7) ? lds32(p0 + 4 + 4 * s) : byte_perm(w0a, w8a, 0x5432u);
      const uint32_t wb = (s < 7) ? lds32(p1 + 4 + 4 * s) : byte_perm(w0b, w8b, 0x5432u);
      const uint32_t xa = lds32(p0 + 36 + 4 * s), xb = lds32(p1 + 36 + 4 * s);
      uint32_t a[4], e[4];
      conv(wa, a[0], a[2]);
      conv(wb, a[1], a[3]);
      conv(xa, e[0], e[2]);
      conv(xb, e[1], e[3]);
      mma_16816(ca, a, B.b[s][0], B.b[s][1]);
      mma_16816(cb, e, B.b[8 + s][0], B.b[8 + s][1]);
    }
    // the halves hold 1152 + q: remove 1152 * (sum of x over the block)
    const float oa = kOffset * sx[2 * L.t], ob = kOffset * sx[2 * L.t + 1];
    tot0 += h_lo(w0a) * ((ca[0] + ca[1]) - oa) + h_hi(w8a) * ((cb[0] + cb[1]) - ob);
    tot1 += h_lo(w0b) * ((ca[2] + ca[3]) - oa) + h_hi(w8b) * ((cb[2] + cb[3]) - ob);
  }
};

struct SegQ4K : Q4K {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const BFrag& B, const float* sx, const LaneCtx& L,
                       float& tot0, float& tot1) {
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
    float cl[4] = {0.f, 0.f, 0.f, 0.f}, ch[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      uint32_t a[4], e[4], t02, t13;
      conv_lo(wa[i], t02, t13);
      a[0] = h2_fma(t02, SL0, CL0);
      a[2] = h2_fma(t13, SL0, CL0);
      conv_lo(wb[i], t02, t13);
      a[1] = h2_fma(t02, SL1, CL1);
      a[3] = h2_fma(t13, SL1, CL1);
      conv_hi(wa[i], t02, t13);
      e[0] = h2_fma(t02, SH0, CH0);
      e[2] = h2_fma(t13, SH0, CH0);
      conv_hi(wb[i], t02, t13);
      e[1] = h2_fma(t02, SH1, CH1);
      e[3] = h2_fma(t13, SH1, CH1);
      mma_16816(cl, a, B.b[2 * i][0], B.b[2 * i][1]);
      mma_16816(ch, e, B.b[2 * i + 1][0], B.b[2 * i + 1][1]);
    }
    const float sxa = sx[j0], sxb = sx[j1];
    const float mt0 = (float)mn00 * sxa + (float)mn01 * sxb;
    const float mt1 = (float)mn10 * sxa + (float)mn11 * sxb;
    tot0 += h_lo(hd0.x) * ((cl[0] + cl[1]) + (ch[0] + ch[1])) - h_hi(hd0.x) * mt0;
    tot1 += h_lo(hd1.x) * ((cl[2] + cl[3]) + (ch[2] + ch[3])) - h_hi(hd1.x) * mt1;
  }
};

struct SegQ6K : Q6K {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const BFrag& B, const float* sx, const LaneCtx& L,
                       float& tot0, float& tot1) {
    const float d0 = __half2float(__ushort_as_half((unsigned short)lds_u16(r0 + 208)));
    const float d1 = __half2float(__ushort_as_half((unsigned short)lds_u16(r1 + 208)));
    const int qlo = 32 * (L.t & 1);
#pragma unroll
    for (int mp = 0; mp < 4; mp += 2) {
      // macro-steps mp (l0 = 0) and mp + 1 (l0 = 16) of half h in two chains
      const int h = mp >> 1;
      uint32_t la[8], ha[8], lb[8], hb[8];
      ld16u(r0 + 64 * h + qlo, *reinterpret_cast<uint32_t(*)[4]>(la));
      ld16u(r0 + 64 * h + qlo + 16, *reinterpret_cast<uint32_t(*)[4]>(la + 4));
      ld16u(r0 + 128 + 32 * h, *reinterpret_cast<uint32_t(*)[4]>(ha));
      ld16u(r0 + 128 + 32 * h + 16, *reinterpret_cast<uint32_t(*)[4]>(ha + 4));
      ld16u(r1 + 64 * h + qlo, *reinterpret_cast<uint32_t(*)[4]>(lb));
      ld16u(r1 + 64 * h + qlo + 16, *reinterpret_cast<uint32_t(*)[4]>(lb + 4));
      ld16u(r1 + 128 + 32 * h, *reinterpret_cast<uint32_t(*)[4]>(hb));
      ld16u(r1 + 128 + 32 * h + 16, *reinterpret_cast<uint32_t(*)[4]>(hb + 4));
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 4; s++) {
        uint32_t a[4], e[4];
        conv(six(la[s], ha[s], L.t), a[0], a[2]);
        conv(six(lb[s], hb[s], L.t), a[1], a[3]);
        conv(six(la[4 + s], ha[4 + s], L.t), e[0], e[2]);
        conv(six(lb[4 + s], hb[4 + s], L.t), e[1], e[3]);
        mma_16816(c0, a, B.b[4 * mp + s][0], B.b[4 * mp + s][1]);
        mma_16816(c1, e, B.b[4 * mp + 4 + s][0], B.b[4 * mp + 4 + s][1]);
      }
      const int gi = 8 * h + 2 * L.t;  // scale group of chain 0 (chain 1: gi + 1)
      const float s00 = (float)lds_s8(r0 + 192 + gi), s01 = (float)lds_s8(r0 + 193 + gi);
      const float s10 = (float)lds_s8(r1 + 192 + gi), s11 = (float)lds_s8(r1 + 193 + gi);
      // the halves hold 1024 + z = (z - 32) + 1056: remove 1056 * group sum
      const float o0 = kOffset * sx[gi], o1 = kOffset * sx[gi + 1];
      tot0 += (d0 * s00) * ((c0[0] + c0[1]) - o0) + (d0 * s01) * ((c1[0] + c1[1]) - o1);
      tot1 += (d1 * s10) * ((c0[2] + c0[3]) - o0) + (d1 * s11) * ((c1[2] + c1[3]) - o1);
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

// B tables of 256-value segments, one warp per segment.  Segment i of the
// source is the fp32 values src[256 i, 256 i + 256), scaled by
// scales[i / segs_per_vec] (a power of two); its table is the 1 KB at
// dst + 1024 i: 16 steps x 4 threads x 16 bytes, the 16-byte chunk c =
// 4 step + t holding f16 hi[4] then f16 lo[4] of elements F::elem(step, t,
// j), j = 0..3.  Its group sums sx[i * 256/GS + g] are the fp32 sums of
// hi + lo over the natural groups of GS = F::kSumGroup values (Q8_0 and
// Q4_K: 32, Q6_K: 16), the offset / min corrections of the segment kernels.
// Every read of a segment precedes every write to it (warp-synchronous), so
// dst may alias src: 4 bytes of table per value, the same footprint.
template <class F>
VDEV void build_tables(const float* src, uint8_t* dst, float* sx, int nseg, int segs_per_vec, const float* scales,
                       int warp, int nwarps, int lane) {
  constexpr int GS = F::kSumGroup;
#pragma unroll 1
  for (int i = warp; i < nseg; i += nwarps) {
    const float sc = scales[i / segs_per_vec];
    const float* v = src + (size_t)i * kSegElems;
    // group sums: lane l holds the natural values [8 l, 8 l + 8)
    const float4 a = *reinterpret_cast<const float4*>(v + 8 * lane);
    const float4 b = *reinterpret_cast<const float4*>(v + 8 * lane + 4);
    const float nat[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const float x = nat[q] * sc;
      const float hi = __half2float(__float2half_rn(x));
      s += hi + __half2float(__float2half_rn(x - hi));
    }
#pragma unroll
    for (int o = 1; o < GS / 8; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    // table chunks c = lane and lane + 32
    uint4 out[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int c = lane + 32 * h, step = c >> 2, t = c & 3;
      uint32_t hv[4], lv[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float x = v[F::elem(step, t, j)] * sc;
        const __half hh = __float2half_rn(x);
        hv[j] = __half_as_ushort(hh);
        lv[j] = __half_as_ushort(__float2half_rn(x - __half2float(hh)));
      }
      out[h] = make_uint4(hv[0] | (hv[1] << 16), hv[2] | (hv[3] << 16), lv[0] | (lv[1] << 16), lv[2] | (lv[3] << 16));
    }
    __syncwarp();
    if ((lane & (GS / 8 - 1)) == 0) sx[(size_t)i * (kSegElems / GS) + lane / (GS / 8)] = s;
    uint4* d4 = reinterpret_cast<uint4*>(dst + (size_t)i * (16 * kStepBytesB));
    d4[lane] = out[0];
    d4[lane + 32] = out[1];
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Consumer side of one unit for warp w: run this warp's segments, reduce each
// over the 4 lanes of a row, publish one 16-row partial per segment, and
// return true in the warp that completes the unit, which sums the segment
// partials in segment order (so the result does not depend on which warp
// computed which segment) into *row_val (lanes 0..15).
// part: [max(nseg, W)][16] floats for this stage.
// ---------------------------------------------------------------------------
template <class S>
VDEV bool consume_unit(const uint8_t* stage, const StageGeom& sg, int v, int nseg, int W, int w,
                       const uint8_t* btab, const float* sx, float* part, int* ucnt, const LaneCtx& L,
                       float* row_val, BFrag& bf) {
  const uint8_t* r0 = stage_row(stage, sg, L.g);
  const uint8_t* r1 = stage_row(stage, sg, L.g + 8);
  int first = (w - (v * nseg) % W) % W;
  if (first < 0) first += W;
#pragma unroll 1
  for (int seg = first; seg < nseg; seg += W) {
    float tot0 = 0.f, tot1 = 0.f;
    bf.get(btab + seg * (16 * kStepBytesB), L);
    S::run(r0 + seg * S::kSegBytes, r1 + seg * S::kSegBytes, bf, sx + seg * (kSegElems / S::kSumGroup), L, tot0,
           tot1);
    tot0 += __shfl_xor_sync(0xffffffffu, tot0, 1);
    tot1 += __shfl_xor_sync(0xffffffffu, tot1, 1);
    tot0 += __shfl_xor_sync(0xffffffffu, tot0, 2);
    tot1 += __shfl_xor_sync(0xffffffffu, tot1, 2);
    if (L.t == 0) {
      part[seg * 16 + L.g] = tot0;
      part[seg * 16 + L.g + 8] = tot1;
    }
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
      for (int seg = 0; seg < nseg; seg++) acc += ((volatile float*)part)[seg * 16 + L.lane];
    *row_val = acc;
    __syncwarp();
    if (L.lane == 0) *ucnt = 0;
  }
  return last != 0;
}

}  // namespace vireo
