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
#pragma unroll 1
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
// B tables of 256-value segments, one warp per segment.  Segment i of the
// source is the fp32 values src[256 i, 256 i + 256).  Its table is the first
// 512 bytes of dst + kSegTabBytes i: step m, thread t, digit c at byte
// 64 m + 16 t + 8 c: the digits of elements F::elem(m, t, r, j) for r = 0, 1
// and j = 0..3.  Its metadata meta[kMeta i ..] holds, per natural 32-value
// group q, the scale s_q = max|x| / 127 and the sum of x~ = s (d1 + d2/254),
// and the same sums per 16-value group.  A group holding inf or NaN gets a
// NaN scale, so that its dot products come out NaN as the reference's do.
// Every read of a segment precedes every write to it (warp-synchronous), so
// dst may alias src (the same 1 KB footprint per segment).
// ---------------------------------------------------------------------------
template <class F>
VDEV void build_tables(const float* src, uint8_t* dst, float* meta, int nseg, int warp, int nwarps, int lane) {
#pragma unroll 1
  for (int i = warp; i < nseg; i += nwarps) {
    const float* v = src + (size_t)i * kSegElems;
    uint8_t* tab = dst + (size_t)i * kSegTabBytes;
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
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    bad = __shfl_xor_sync(0xffffffffu, (int)bad, 1) | __shfl_xor_sync(0xffffffffu, (int)bad, 2) | bad;
    const float sc = bad ? __int_as_float(0x7fc00000) : mx * (1.0f / 127.0f);
    const float inv = (mx > 0.f && !bad) ? 127.0f / mx : 0.f;
    uint32_t lo1 = 0, hi1 = 0, lo2 = 0, hi2 = 0;
    int s1 = 0, s2 = 0;
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const float y = x[q] * inv;
      const float r1 = fminf(fmaxf(rintf(y), -127.f), 127.f);
      const float r2 = fminf(fmaxf(rintf((y - r1) * 254.f), -127.f), 127.f);
      const int i1 = (int)r1, i2 = (int)r2;
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
    // sums of x~ per 16-group (lane pairs) and per 32-group (lane quads)
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
    const float sum16 = sc * ((float)s1 + (float)s2 * kInv254);
    const int t1 = s1 + __shfl_xor_sync(0xffffffffu, s1, 2), t2 = s2 + __shfl_xor_sync(0xffffffffu, s2, 2);
    const float sum32 = sc * ((float)t1 + (float)t2 * kInv254);
    __syncwarp();  // every lane holds its values: the segment may be overwritten
    // natural-order digits in the scratch half: d1 at +512, d2 at +768
    *reinterpret_cast<uint2*>(tab + 512 + 8 * lane) = make_uint2(lo1, hi1);
    *reinterpret_cast<uint2*>(tab + 768 + 8 * lane) = make_uint2(lo2, hi2);
    if ((lane & 3) == 0) {
      meta[(size_t)i * kMeta + lane / 4] = sc;
      meta[(size_t)i * kMeta + 8 + lane / 4] = sum32;
    }
    if ((lane & 1) == 0) meta[(size_t)i * kMeta + 16 + lane / 2] = sum16;
    __syncwarp();
    // table chunks ch = lane, lane + 32: step m = ch >> 3, thread t = (ch >> 1) & 3, digit c = ch & 1
    uint2 out[2];
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
      out[hh] = make_uint2(w[0], w[1]);
    }
    __syncwarp();
    reinterpret_cast<uint2*>(tab)[lane] = out[0];
    reinterpret_cast<uint2*>(tab)[lane + 32] = out[1];
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
                       const uint8_t* btab, const float* meta, float* part, int* ucnt, const LaneCtx& L,
                       float* row_val, BFrag& bf) {
  const uint8_t* r0 = stage_row(stage, sg, L.g);
  const uint8_t* r1 = stage_row(stage, sg, L.g + 8);
  int first = (w - (v * nseg) % W) % W;
  if (first < 0) first += W;
#pragma unroll 1
  for (int seg = first; seg < nseg; seg += W) {
    float tot0 = 0.f, tot1 = 0.f;
    bf.get(btab + seg * kSegTabBytes, L);
    S::run(r0 + seg * S::kSegBytes, r1 + seg * S::kSegBytes, bf, meta + seg * kMeta, L, tot0, tot1);
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
