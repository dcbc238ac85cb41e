// GGUF block formats -> integer tensor-core fragments.
//
// The decode GEMV multiplies 16-row weight tiles by one activation vector
// with mma.sync.m16n8k32 (int8 x int8 -> int32).  Weights are the A operand,
// read straight from the raw GGUF bytes staged in shared memory: Q8_0 quants
// as s8, Q4_K nibbles and Q6_K 6-bit values as u8, only masked in place.
// The activation vector is the B operand: for each natural 32-value group a
// scale s = max|x| / 127 and two int8 digits per value, x ~ s (d1 + d2/254)
// (|error| <= s / 508, about 1.6e-5 of the group's largest value).
//
// Fragment layout of m16n8k32 (lane = 4 g + t): A registers {row g, k 4t..
// 4t+3}, {row g+8, same k}, {row g, k 16+4t..}, {row g+8, k 16+4t..}; B
// registers {k 4t.., column g}, {k 16+4t.., column g}; C {row g: columns 2t,
// 2t+1}, {row g+8: columns 2t, 2t+1}.  The order of k inside a step is free
// as long as A and B agree, so each format maps thread t's k-slots to 8 of
// its OWN values (all in one scale group).  "Column trick": B column 2t
// holds d1 and column 2t+1 holds d2, only at thread t's k-slots, so lane
// (g, t) ends a run of steps holding in C[2t], C[2t+1] the exact integer
// dot products over the values it supplied, and applies its own block
// scales in fp32.
//
// A segment is 256 consecutive values of a row: 8 steps of k32, thread t
// supplying 64 values.  F::elem(m, t, r, j) is the segment value behind step
// m, thread t, register r (0: k 4t+j, 1: k 16+4t+j), byte j.
//
// Reference block layouts: vireo src/gguf_compute.c:38-42 (structs),
// :45-51 (Q4_K scale/min packing), :52-66 (Q4_K), :83-103 (Q6_K).
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define VHD __host__ __device__ __forceinline__
#else
#define VHD inline
#endif

namespace vireo {

enum : uint32_t { T_F32 = 0, T_F16 = 1, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

constexpr int kSegElems = 256;   // every fast-path format works in 256-value segments
constexpr int kSegSteps = 8;     // k32 tensor-core steps per segment
constexpr int kStepBytesB = 64;  // B table bytes per step: [t][digit][2 regs x 4 x int8]
constexpr int kSegTabBytes = 1024;  // B table stride per segment (512 used, 512 build scratch)
constexpr int kMeta = 36;        // floats of per-segment activation metadata:
                                 // [0,8) scale of each 32-group, [8,16) sum of x~ per
                                 // 32-group, [16,32) sum of x~ per 16-group, [32] residual
                                 // table flag, [33,36) padding
constexpr int kMetaFlag = 32;

// ---- portable bit helpers (host versions for the self-test) --------------
// 3-input bitwise function with lookup table lut (a, b, c <-> 0xF0, 0xCC, 0xAA)
#ifdef __CUDA_ARCH__
template <uint32_t LUT>
__device__ __forceinline__ uint32_t lop3t(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
  return d;
}
#else
template <uint32_t LUT>
inline uint32_t lop3t(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d = 0;
  for (int i = 0; i < 32; i++) {
    uint32_t idx = (((a >> i) & 1u) << 2) | (((b >> i) & 1u) << 1) | ((c >> i) & 1u);
    d |= ((LUT >> idx) & 1u) << i;
  }
  return d;
}
#endif
VHD uint32_t byte_perm(uint32_t a, uint32_t b, uint32_t s) {
#ifdef __CUDA_ARCH__
  return __byte_perm(a, b, s);
#else
  uint64_t x = ((uint64_t)b << 32) | a;
  uint32_t r = 0;
  for (int i = 0; i < 4; i++) {
    uint32_t sel = (s >> (4 * i)) & 7u;
    r |= (uint32_t)((x >> (8 * sel)) & 0xFFu) << (8 * i);
  }
  return r;
#endif
}

// ---- Q8_0: 34-byte blocks (f16 d, 32 x int8), segment = 8 blocks --------
// Thread t owns the block pair (2t, 2t+1) = bytes [68t, 68t+68) of the
// segment, 17 aligned words: W0 = [dA dA q0 q1], W1..W7 = q2..q29,
// W8 = [q30 q31 dB dB], W9..W16 = block B's 32 quants.  Steps 0..3 cover
// block A with (W1, W2), (W3, W4), (W5, W6), (W7, [q0 q1 q30 q31] = prmt(W0,
// W8)); steps 4..7 cover block B with (W9, W10) .. (W15, W16).  The quants
// are the s8 A operand as they are.
struct Q8 {
  static constexpr uint32_t kType = T_Q8_0;
  static constexpr int kSegBytes = 272;
  VHD static int elem(int m, int t, int r, int j) {
    const int base = 64 * t;
    if (m >= 4) return base + 32 + 8 * (m - 4) + 4 * r + j;
    if (m < 3 || r == 0) return base + 4 * (1 + 2 * m + r) - 2 + j;
    return base + (j < 2 ? j : 28 + j);
  }
};

// ---- Q5_0: 22-byte blocks (f16 d, 4 bytes qh, 16 bytes qs), segment = 8
// blocks.  Value j of a block (reference dequant_row_q5_0, gguf_compute.c:
// 68-82): q = (j < 16 ? qs[j] & 15 : qs[j - 16] >> 4) | (bit j of qh) << 4,
// value = d (q - 16).  Thread t owns the block pair (2t, 2t+1) = bytes [44t,
// 44t + 44) of the segment, 11 aligned words: W0 = [dA dA qhA qhA], W1 =
// [qhA qhA qs0 qs1], .., W5 = [qs14 qs15 dB dB], W6 = qhB, W7..W10 = block
// B's qs.  Steps 0..3 cover block 2t (values 8 m + 4 r + j), steps 4..7
// block 2t+1.  The u8 q values are the A operand; the 16 is removed with the
// 32-group sum of x.
struct Q5 {
  static constexpr uint32_t kType = T_Q5_0;
  static constexpr int kSegBytes = 176;
  VHD static int elem(int m, int t, int r, int j) { return 64 * t + 8 * m + 4 * r + j; }
};

// ---- Q4_K: 144-byte super-blocks, segment = 1 super-block ---------------
// Thread t owns the 64-value chunk t: the 32 bytes qs[32t, 32t+32) as words
// w0..w7; byte l's low nibble is value 64t + l (sub-block 2t), its high
// nibble value 64t + 32 + l (sub-block 2t+1).  Steps 0..3: low nibbles of
// (w[2m], w[2m+1]) (w & 0x0F0F0F0F, u8 q); steps 4..7: high nibbles of
// (w[2m-8], w[2m-7]) as u8 16q (w & 0xF0F0F0F0, the 1/16 goes to the
// scale).  Value = d sc_j q - dmin m_j; the min term is applied with the
// group sum of x.
struct Q4K {
  static constexpr uint32_t kType = T_Q4_K;
  static constexpr int kSegBytes = 144;
  VHD static int elem(int m, int t, int r, int j) { return 64 * t + (m >= 4 ? 32 : 0) + 8 * (m & 3) + 4 * r + j; }
  // 6-bit (scale, min) of sub-block j from the 12 packed bytes held in
  // three little-endian words S0 = bytes 0..3, S1 = 4..7, S2 = 8..11.
  VHD static void scale_min(uint32_t S0, uint32_t S1, uint32_t S2, int j, uint32_t& sc, uint32_t& mn) {
    uint32_t sh = 8u * (uint32_t)(j & 3);
    uint32_t b0 = (S0 >> sh) & 0xFFu, b1 = (S1 >> sh) & 0xFFu, b2 = (S2 >> sh) & 0xFFu;
    uint32_t sl = b0 & 63u, ml = b1 & 63u;
    uint32_t shh = (b2 & 15u) | ((b0 >> 6) << 4), mh = (b2 >> 4) | ((b1 >> 6) << 4);
    sc = (j < 4) ? sl : shh;
    mn = (j < 4) ? ml : mh;
  }
};

// ---- Q6_K: 210-byte super-blocks, segment = 1 super-block ---------------
// Thread t follows stream t of each half h (reference q1..q4): value 128h +
// 32t + l has its low 4 bits in the low (t < 2) or high (t >= 2) nibble of
// ql[64h + 32(t&1) + l] and its top 2 bits in bits (2t, 2t+1) of
// qh[32h + l]; int8 scale sc[8h + 2t + l/16].  Step m: h = m >> 2, l = 16
// ((m >> 1) & 1) + 8 (m & 1) + 4r + j, so each pair of steps is one 16-value
// scale group.  z = the 6-bit value as u8; value = d sc (z - 32), the 32 is
// removed with the 16-group sum of x.  Super-blocks are only 2-byte aligned
// in general (210 = 2 mod 4): words are read with a funnel shift.
struct Q6K {
  static constexpr uint32_t kType = T_Q6_K;
  static constexpr int kSegBytes = 210;
  VHD static int elem(int m, int t, int r, int j) {
    return 128 * (m >> 2) + 32 * t + 16 * ((m >> 1) & 1) + 8 * (m & 1) + 4 * r + j;
  }
  // 4 six-bit values of stream t from a ql word and a qh word
  VHD static uint32_t six(uint32_t ql, uint32_t qh, int t) {
    uint32_t lo = (ql >> (4u * (uint32_t)(t >> 1))) & 0x0F0F0F0Fu;
    uint32_t hi = ((qh >> (2u * (uint32_t)t)) & 0x03030303u) << 4;
    return lo | hi;
  }
};

}  // namespace vireo
