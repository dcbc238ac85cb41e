// Streaming dequant-GEMV engine shared by the decode kernels.
//
// Work is cut into tiles of 16 weight rows x full K.  One producer warp moves
// the raw GGUF rows of each item (one or more tiles) from HBM into a ring of
// shared-memory stages with 1-D bulk copies (cp.async.bulk: one instruction
// per row or per group of rows, executed by the TMA engine, completing on the
// stage's mbarrier; never multicast).  The consumer warps run the
// tensor-core segment kernels below over each tile's 256-value segments:
// the MoE kernel gives a whole tile to one warp, or to a warp pair that
// splits its segments (segments in order, in registers); the stand-alone
// GEMV deals a tile's segments over the warps
// (consume_unit) and the warp that completes the tile sums the segment
// partials in segment order.  Either way the result does not depend on
// which warp computed what.
//
// Stage layout: rows 0..7 ("half 0") and 8..15 ("half 1") may come from
// different matrices (gate and up rows of one expert).  Rows are copied in
// dense groups of G rows, one bulk copy per group, the groups padded to
// start 16 B apart modulo 128 B (stage_geom picks G per format and row
// size so that the lanes of a warp spread over the banks).
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
};

VDEV const uint8_t* stage_row(const uint8_t* stage, const StageGeom& sg, int r) {
  int h = r >> 3, r8 = r & 7;
  return stage + h * sg.hstride + (r8 / (int)sg.G) * sg.gstride + (r8 % (int)sg.G) * sg.rb;
}

// Producer side: one tile (16 rows) of bulk copies, issued by lanes
// 0 .. 2 (8 / G) - 1 of the calling warp (one copy per row or row group).
// The caller has already announced the item's bytes on `full` with
// mbar_arrive_expect_tx (16 rb per tile); each copy completes its bytes on
// it.  Source and destination addresses and sizes are multiples of 16.
VDEV void issue_tile_bulk(uint8_t* stage, uint64_t* full, const uint8_t* src0, const uint8_t* src1,
                          const StageGeom& sg, int lane) {
  const int groups = 8 / (int)sg.G;
  if (lane < 2 * groups) {
    const int h = lane >= groups ? 1 : 0, j = lane - h * groups;
    const uint32_t gbytes = sg.G * sg.rb;
    bulk_g2s(stage + h * sg.hstride + j * sg.gstride, (h ? src1 : src0) + (size_t)j * gbytes, gbytes, full);
  }
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
// B fragments of one segment held in registers (8 steps x 2 regs); a warp
// that meets the same segment of the same table again (consecutive units
// whose segment index lands on the same warp) skips the reload.
// ---------------------------------------------------------------------------
struct BFrag {
  uint32_t b[kSegSteps][2];
  const uint8_t* key;
  VDEV void reset() { key = nullptr; }
  VDEV void get(const uint8_t* segtab, const LaneCtx& L) {
    if (segtab == key) return;
    key = segtab;
#pragma unroll
    for (int s = 0; s < kSegSteps; s++) {
      const uint2 v = lds64(segtab + s * kStepBytesB + L.boff);
      b[s][0] = L.bon ? v.x : 0u;
      b[s][1] = L.bon ? v.y : 0u;
    }
  }
};

constexpr float kInv254 = 1.0f / 254.0f;
// s * (d1-dot + d2-dot / 254) for one C column pair
VDEV float dig(int c0, int c1) { return (float)c0 + (float)c1 * kInv254; }

// ---------------------------------------------------------------------------
// Segment kernels: accumulate one 256-value segment of rows g (r0) and g+8
// (r1) into this lane's fp32 totals.  B: the segment's fragments; meta: the
// segment's activation metadata (kMeta floats).  Independent scale groups
// run as independent accumulator chains.
// ---------------------------------------------------------------------------
struct SegQ8 : Q8 {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const BFrag& B, const float* meta, const LaneCtx& L,
                       float& tot0, float& tot1) {
    const uint8_t* p0 = r0 + 68 * L.t;
    const uint8_t* p1 = r1 + 68 * L.t;
    uint32_t wa[17], wb[17];
#pragma unroll
    for (int i = 0; i < 17; i++) {
      wa[i] = lds32(p0 + 4 * i);
      wb[i] = lds32(p1 + 4 * i);
    }
    int ca[4], cb[4];
#pragma unroll
    for (int m = 0; m < 4; m++) {
      uint32_t a[4], e[4];
      a[0] = wa[1 + 2 * m];
      a[1] = wb[1 + 2 * m];
      a[2] = (m < 3) ? wa[2 + 2 * m] : byte_perm(wa[0], wa[8], 0x5432u);
      a[3] = (m < 3) ? wb[2 + 2 * m] : byte_perm(wb[0], wb[8], 0x5432u);
      e[0] = wa[9 + 2 * m];
      e[1] = wb[9 + 2 * m];
      e[2] = wa[10 + 2 * m];
      e[3] = wb[10 + 2 * m];
      if (m == 0) {
        imma_s8_z(ca, a, B.b[0][0], B.b[0][1]);
        imma_s8_z(cb, e, B.b[4][0], B.b[4][1]);
      } else {
        imma_s8(ca, a, B.b[m][0], B.b[m][1]);
        imma_s8(cb, e, B.b[4 + m][0], B.b[4 + m][1]);
      }
    }
    const float sA = meta[2 * L.t], sB = meta[2 * L.t + 1];
    tot0 += h_lo(wa[0]) * sA * dig(ca[0], ca[1]) + h_hi(wa[8]) * sB * dig(cb[0], cb[1]);
    tot1 += h_lo(wb[0]) * sA * dig(ca[2], ca[3]) + h_hi(wb[8]) * sB * dig(cb[2], cb[3]);
  }
};

// The u8 values v .. v+3 (v a multiple of 4) of a Q5_0 block from its qs
// words and qh: low or high nibbles, bit v + i of qh as bit 4 of byte i (the
// multiply spreads four bits to bytes 0..3 without carries).
VDEV uint32_t q5_four(const uint32_t (&qs)[4], uint32_t qh, int v) {
  const uint32_t nib = (qs[(v & 15) >> 2] >> (v >= 16 ? 4 : 0)) & 0x0F0F0F0Fu;
  const uint32_t hb = ((((qh >> v) & 0xFu) * 0x00204081u) & 0x01010101u) << 4;
  return nib | hb;
}

struct SegQ5 : Q5 {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const BFrag& B, const float* meta, const LaneCtx& L,
                       float& tot0, float& tot1) {
    const uint8_t* p0 = r0 + 44 * L.t;
    const uint8_t* p1 = r1 + 44 * L.t;
    uint32_t wa[11], wb[11];
#pragma unroll
    for (int i = 0; i < 11; i++) {
      wa[i] = lds32(p0 + 4 * i);
      wb[i] = lds32(p1 + 4 * i);
    }
    const uint32_t qha = __funnelshift_r(wa[0], wa[1], 16), qhb = __funnelshift_r(wb[0], wb[1], 16);
    const uint32_t sa[4] = {__funnelshift_r(wa[1], wa[2], 16), __funnelshift_r(wa[2], wa[3], 16),
                            __funnelshift_r(wa[3], wa[4], 16), __funnelshift_r(wa[4], wa[5], 16)};
    const uint32_t sb[4] = {__funnelshift_r(wb[1], wb[2], 16), __funnelshift_r(wb[2], wb[3], 16),
                            __funnelshift_r(wb[3], wb[4], 16), __funnelshift_r(wb[4], wb[5], 16)};
    const uint32_t ta[4] = {wa[7], wa[8], wa[9], wa[10]}, tb[4] = {wb[7], wb[8], wb[9], wb[10]};
    int ca[4], cb[4];
#pragma unroll
    for (int m = 0; m < 4; m++) {
      uint32_t a[4], e[4];
      a[0] = q5_four(sa, qha, 8 * m);
      a[1] = q5_four(sb, qhb, 8 * m);
      a[2] = q5_four(sa, qha, 8 * m + 4);
      a[3] = q5_four(sb, qhb, 8 * m + 4);
      e[0] = q5_four(ta, wa[6], 8 * m);
      e[1] = q5_four(tb, wb[6], 8 * m);
      e[2] = q5_four(ta, wa[6], 8 * m + 4);
      e[3] = q5_four(tb, wb[6], 8 * m + 4);
      if (m == 0) {
        imma_u8_z(ca, a, B.b[0][0], B.b[0][1]);
        imma_u8_z(cb, e, B.b[4][0], B.b[4][1]);
      } else {
        imma_u8(ca, a, B.b[m][0], B.b[m][1]);
        imma_u8(cb, e, B.b[4 + m][0], B.b[4 + m][1]);
      }
    }
    const int ga = 2 * L.t, gb = 2 * L.t + 1;
    const float sA = meta[ga], sB = meta[gb], SA = 16.f * meta[8 + ga], SB = 16.f * meta[8 + gb];
    tot0 += h_lo(wa[0]) * (sA * dig(ca[0], ca[1]) - SA) + h_hi(wa[5]) * (sB * dig(cb[0], cb[1]) - SB);
    tot1 += h_lo(wb[0]) * (sA * dig(ca[2], ca[3]) - SA) + h_hi(wb[5]) * (sB * dig(cb[2], cb[3]) - SB);
  }
};

struct SegQ4K : Q4K {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const BFrag& B, const float* meta, const LaneCtx& L,
                       float& tot0, float& tot1) {
    const uint4 hd0 = lds128(r0), hd1 = lds128(r1);
    const uint4 qa0 = lds128(r0 + 16 + 32 * L.t), qa1 = lds128(r0 + 32 + 32 * L.t);
    const uint4 qb0 = lds128(r1 + 16 + 32 * L.t), qb1 = lds128(r1 + 32 + 32 * L.t);
    const uint32_t wa[8] = {qa0.x, qa0.y, qa0.z, qa0.w, qa1.x, qa1.y, qa1.z, qa1.w};
    const uint32_t wb[8] = {qb0.x, qb0.y, qb0.z, qb0.w, qb1.x, qb1.y, qb1.z, qb1.w};
    int cl[4], ch[4];
#pragma unroll
    for (int m = 0; m < 4; m++) {
      uint32_t a[4], e[4];
      a[0] = wa[2 * m] & 0x0F0F0F0Fu;
      a[1] = wb[2 * m] & 0x0F0F0F0Fu;
      a[2] = wa[2 * m + 1] & 0x0F0F0F0Fu;
      a[3] = wb[2 * m + 1] & 0x0F0F0F0Fu;
      e[0] = wa[2 * m] & 0xF0F0F0F0u;
      e[1] = wb[2 * m] & 0xF0F0F0F0u;
      e[2] = wa[2 * m + 1] & 0xF0F0F0F0u;
      e[3] = wb[2 * m + 1] & 0xF0F0F0F0u;
      if (m == 0) {
        imma_u8_z(cl, a, B.b[0][0], B.b[0][1]);
        imma_u8_z(ch, e, B.b[4][0], B.b[4][1]);
      } else {
        imma_u8(cl, a, B.b[m][0], B.b[m][1]);
        imma_u8(ch, e, B.b[4 + m][0], B.b[4 + m][1]);
      }
    }
    const int j0 = 2 * L.t, j1 = 2 * L.t + 1;
    uint32_t sc00, mn00, sc01, mn01, sc10, mn10, sc11, mn11;
    scale_min(hd0.y, hd0.z, hd0.w, j0, sc00, mn00);
    scale_min(hd0.y, hd0.z, hd0.w, j1, sc01, mn01);
    scale_min(hd1.y, hd1.z, hd1.w, j0, sc10, mn10);
    scale_min(hd1.y, hd1.z, hd1.w, j1, sc11, mn11);
    const float s0 = meta[j0], s1 = meta[j1] * 0.0625f;  // high nibbles were 16 q
    const float S0 = meta[8 + j0], S1 = meta[8 + j1];
    tot0 += h_lo(hd0.x) * ((float)sc00 * s0 * dig(cl[0], cl[1]) + (float)sc01 * s1 * dig(ch[0], ch[1])) -
            h_hi(hd0.x) * ((float)mn00 * S0 + (float)mn01 * S1);
    tot1 += h_lo(hd1.x) * ((float)sc10 * s0 * dig(cl[2], cl[3]) + (float)sc11 * s1 * dig(ch[2], ch[3])) -
            h_hi(hd1.x) * ((float)mn10 * S0 + (float)mn11 * S1);
  }
};

struct SegQ6K : Q6K {
  VDEV static void run(const uint8_t* r0, const uint8_t* r1, const BFrag& B, const float* meta, const LaneCtx& L,
                       float& tot0, float& tot1) {
    const float d0 = __half2float(__ushort_as_half((unsigned short)lds_u16(r0 + 208)));
    const float d1 = __half2float(__ushort_as_half((unsigned short)lds_u16(r1 + 208)));
    const int qlo = 32 * (L.t & 1);
#pragma unroll
    for (int q = 0; q < 4; q++) {
      // scale group q: half h = q >> 1, l0 = 16 (q & 1); steps 2q, 2q + 1
      const int h = q >> 1, l0 = 16 * (q & 1);
      uint32_t la[4], ha[4], lb[4], hb[4];
      ld16u(r0 + 64 * h + qlo + l0, la);
      ld16u(r0 + 128 + 32 * h + l0, ha);
      ld16u(r1 + 64 * h + qlo + l0, lb);
      ld16u(r1 + 128 + 32 * h + l0, hb);
      uint32_t a[4], e[4];
      a[0] = six(la[0], ha[0], L.t);
      a[1] = six(lb[0], hb[0], L.t);
      a[2] = six(la[1], ha[1], L.t);
      a[3] = six(lb[1], hb[1], L.t);
      e[0] = six(la[2], ha[2], L.t);
      e[1] = six(lb[2], hb[2], L.t);
      e[2] = six(la[3], ha[3], L.t);
      e[3] = six(lb[3], hb[3], L.t);
      int c[4];
      imma_u8_z(c, a, B.b[2 * q][0], B.b[2 * q][1]);
      imma_u8(c, e, B.b[2 * q + 1][0], B.b[2 * q + 1][1]);
      const int gi = 8 * h + 2 * L.t + (q & 1);  // scale index = 16-group index
      const float xs = meta[4 * h + L.t], S16 = 32.f * meta[16 + gi];
      tot0 += d0 * (float)lds_s8(r0 + 192 + gi) * (xs * dig(c[0], c[1]) - S16);
      tot1 += d1 * (float)lds_s8(r1 + 192 + gi) * (xs * dig(c[2], c[3]) - S16);
    }
  }
};

// ---------------------------------------------------------------------------
// Activation tables.  Segment i of a vector is its values [256 i, 256 i +
// 256).  Its B table is the first 512 bytes of tab + kSegTabBytes i: step m,
// thread t, digit c at byte 64 m + 16 t + 8 c: the digits of elements
// F::elem(m, t, r, j) for r = 0, 1 and j = 0..3.  Its metadata meta[kMeta i
// ..] holds, per natural 32-value group q, the scale s_q = max|x| / 127 and
// the sum of x~ = s (d1 + d2/254), the same sums per 16-value group, and at
// kMetaFlag whether the segment has a residual table.
//
// Residual tables: the two digits leave an error of up to max|x| / 64516 on
// every value of a group, which is small against the group's own values
// unless one value dwarfs the others (an outlier channel).  A segment in
// which some group's largest magnitude exceeds kResRatio times the median of
// the segment's eight group maxima gets a second table of the same form for
// the remainder
// r = x - x~ (rtab + kResTabBytes i, rmeta + kMeta i); the consumers add the
// products with it, so every value of such a segment is carried to about
// max|x| / 64516^2.  The dot products are linear in the activations, so the
// segment kernels run unchanged on the second table.
//
// A group holding inf or NaN gets a NaN scale (and no residual table), so
// that its dot products come out NaN as the reference's do.  Every read of a
// segment's source precedes every write to its table (warp-synchronous), so
// the source may alias tab (the same 1 KB footprint per segment).
// ---------------------------------------------------------------------------
constexpr int kResTabBytes = 512;
constexpr float kResRatio = 4.0f;

struct VecTab {
  uint8_t* tab;   // [nseg][kSegTabBytes]
  float* meta;    // [nseg][kMeta]
  uint8_t* rtab;  // [nseg][kResTabBytes]
  float* rmeta;   // [nseg][kMeta]
};

// Two int8 digits of 8 values under scale 1 / inv (inv = 0: all zero):
// packed natural-order bytes of digit 1 (lo1 | hi1) and digit 2, and their
// sums over the 8 values.
VDEV void digits8(const float (&x)[8], float inv, uint32_t& lo1, uint32_t& hi1, uint32_t& lo2, uint32_t& hi2,
                  int& s1, int& s2, float (&used)[8]) {
  lo1 = hi1 = lo2 = hi2 = 0;
  s1 = s2 = 0;
#pragma unroll
  for (int q = 0; q < 8; q++) {
    const float y = x[q] * inv;
    const float r1 = fminf(fmaxf(rintf(y), -127.f), 127.f);
    const float r2 = fminf(fmaxf(rintf((y - r1) * 254.f), -127.f), 127.f);
    const int i1 = (int)r1, i2 = (int)r2;
    used[q] = r1 + r2 * kInv254;
    s1 += i1;
    s2 += i2;
    const uint32_t b1 = (uint32_t)(i1 & 0xFF), b2 = (uint32_t)(i2 & 0xFF);
    if (q < 4) {
      lo1 |= b1 << (8 * q);
      lo2 |= b2 << (8 * q);
    } else {
      hi1 |= b1 << (8 * (q - 4));
      hi2 |= b2 << (8 * (q - 4));
    }
  }
}

// Natural-order digits (8 bytes per lane per digit) through the scratch half
// of tab into the step layout, written to out (512 bytes).  Warp-collective.
template <class F>
VDEV void digits_to_table(uint8_t* tab, uint8_t* out, int lane, uint32_t lo1, uint32_t hi1, uint32_t lo2,
                          uint32_t hi2) {
  __syncwarp();
  *reinterpret_cast<uint2*>(tab + 512 + 8 * lane) = make_uint2(lo1, hi1);
  *reinterpret_cast<uint2*>(tab + 768 + 8 * lane) = make_uint2(lo2, hi2);
  __syncwarp();
  // table chunks ch = lane, lane + 32: step m = ch >> 3, thread t = (ch >> 1) & 3, digit c = ch & 1
  uint2 o[2];
#pragma unroll
  for (int hh = 0; hh < 2; hh++) {
    const int ch = lane + 32 * hh, m = ch >> 3, t = (ch >> 1) & 3, c = ch & 1;
    const uint8_t* nat = tab + 512 + 256 * c;
    uint32_t w[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
      uint32_t acc = 0;
#pragma unroll
      for (int j = 0; j < 4; j++) acc |= (uint32_t)nat[F::elem(m, t, r, j)] << (8 * j);
      w[r] = acc;
    }
    o[hh] = make_uint2(w[0], w[1]);
  }
  __syncwarp();
  reinterpret_cast<uint2*>(out)[lane] = o[0];
  reinterpret_cast<uint2*>(out)[lane + 32] = o[1];
  __syncwarp();
}

// Per-group scale and metadata sums of one digit pair: lane l holds 8 values
// of 32-group l / 4; meta gets s, the 32-group sum and the 16-group sum.
VDEV void group_meta(float* meta, int lane, float sc, int s1, int s2) {
  s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
  s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
  const float sum16 = sc * ((float)s1 + (float)s2 * kInv254);
  const int t1 = s1 + __shfl_xor_sync(0xffffffffu, s1, 2), t2 = s2 + __shfl_xor_sync(0xffffffffu, s2, 2);
  const float sum32 = sc * ((float)t1 + (float)t2 * kInv254);
  if ((lane & 3) == 0) {
    meta[lane / 4] = sc;
    meta[8 + lane / 4] = sum32;
  }
  if ((lane & 1) == 0) meta[16 + lane / 2] = sum16;
}

VDEV float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

template <class F>
VDEV void build_tables(const float* src, const VecTab& T, int nseg, int warp, int nwarps, int lane) {
#pragma unroll 1
  for (int i = warp; i < nseg; i += nwarps) {
    const float* v = src + (size_t)i * kSegElems;
    uint8_t* tab = T.tab + (size_t)i * kSegTabBytes;
    float* meta = T.meta + (size_t)i * kMeta;
    // lane l holds the natural values [8 l, 8 l + 8): 32-group l / 4
    const float4 a4 = *reinterpret_cast<const float4*>(v + 8 * lane);
    const float4 b4 = *reinterpret_cast<const float4*>(v + 8 * lane + 4);
    const float x[8] = {a4.x, a4.y, a4.z, a4.w, b4.x, b4.y, b4.z, b4.w};
    float mx = 0.f;
    bool bad = false;
#pragma unroll
    for (int q = 0; q < 8; q++) {
      mx = fmaxf(mx, fabsf(x[q]));
      bad |= !(fabsf(x[q]) <= 3.402823466e38f);
    }
    mx = quad_max(mx);
    bad = __shfl_xor_sync(0xffffffffu, (int)bad, 1) | __shfl_xor_sync(0xffffffffu, (int)bad, 2) | bad;
    const float sc = bad ? __int_as_float(0x7fc00000) : mx * (1.0f / 127.0f);
    const float inv = (mx > 0.f && !bad) ? 127.0f / mx : 0.f;
    uint32_t lo1, hi1, lo2, hi2;
    int s1, s2;
    float used[8];
    digits8(x, inv, lo1, hi1, lo2, hi2, s1, s2, used);
    // an outlier group: its max above kResRatio x the median (the mean of
    // the 4th and 5th smallest) of the segment's 8 group maxima; finite
    // segments only
    float gm[8];
#pragma unroll
    for (int k = 0; k < 8; k++) gm[k] = __shfl_sync(0xffffffffu, mx, 4 * k);
#pragma unroll
    for (int a = 1; a < 8; a++)
#pragma unroll
      for (int b = a; b > 0; b--) {
        const float lo = fminf(gm[b - 1], gm[b]), hi = fmaxf(gm[b - 1], gm[b]);
        gm[b - 1] = lo;
        gm[b] = hi;
      }
    const bool seg_bad = __any_sync(0xffffffffu, bad);
    const bool flagged = !seg_bad && gm[7] > kResRatio * 0.5f * (gm[3] + gm[4]);
    group_meta(meta, lane, sc, s1, s2);
    digits_to_table<F>(tab, tab, lane, lo1, hi1, lo2, hi2);
    if (flagged) {
      float r[8];
#pragma unroll
      for (int q = 0; q < 8; q++) r[q] = bad ? 0.f : x[q] - sc * used[q];
      float mr = 0.f;
#pragma unroll
      for (int q = 0; q < 8; q++) mr = fmaxf(mr, fabsf(r[q]));
      mr = quad_max(mr);
      const float scr = mr * (1.0f / 127.0f), invr = mr > 0.f ? 127.0f / mr : 0.f;
      digits8(r, invr, lo1, hi1, lo2, hi2, s1, s2, used);
      group_meta(T.rmeta + (size_t)i * kMeta, lane, scr, s1, s2);
      digits_to_table<F>(tab, T.rtab + (size_t)i * kResTabBytes, lane, lo1, hi1, lo2, hi2);
    }
    if (lane == 0) meta[kMetaFlag] = flagged ? 1.f : 0.f;
  }
}

// One segment of rows g (r0) and g + 8 (r1) of a tile against a vector's
// tables, both passes (main table, and the residual table when the segment
// has one), accumulated into this lane's totals.
template <class SF>
VDEV void seg_dot(const uint8_t* r0, const uint8_t* r1, int seg, const VecTab& T, const LaneCtx& L, BFrag& bf,
                  float& tot0, float& tot1) {
  const int passes = T.meta[(size_t)seg * kMeta + kMetaFlag] != 0.f ? 2 : 1;
#pragma unroll 1
  for (int ps = 0; ps < passes; ps++) {
    bf.get(ps ? T.rtab + (size_t)seg * kResTabBytes : T.tab + (size_t)seg * kSegTabBytes, L);
    SF::run(r0 + seg * SF::kSegBytes, r1 + seg * SF::kSegBytes, bf, (ps ? T.rmeta : T.meta) + (size_t)seg * kMeta,
            L, tot0, tot1);
  }
}

// ---------------------------------------------------------------------------
// Consumer side of one tile for warp w: run this warp's segments, reduce each
// over the 4 lanes of a row, publish one 16-row partial per segment, and
// return true in the warp that completes the tile, which sums the segment
// partials in segment order (so the result does not depend on which warp
// computed which segment) into *row_val (lanes 0..15).
// part: [max(nseg, W)][16] floats for this stage.
// ---------------------------------------------------------------------------
template <class S>
VDEV bool consume_unit(const uint8_t* stage, const StageGeom& sg, int v, int nseg, int W, int w, const VecTab& T,
                       float* part, int* ucnt, const LaneCtx& L, float* row_val, BFrag& bf) {
  const uint8_t* r0 = stage_row(stage, sg, L.g);
  const uint8_t* r1 = stage_row(stage, sg, L.g + 8);
  int first = (w - (v * nseg) % W) % W;
  if (first < 0) first += W;
#pragma unroll 1
  for (int seg = first; seg < nseg; seg += W) {
    float tot0 = 0.f, tot1 = 0.f;
    seg_dot<S>(r0, r1, seg, T, L, bf, tot0, tot1);
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
