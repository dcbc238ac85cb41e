// GGUF block formats -> tensor-core fragments.
//
// The decode GEMV multiplies a 16-row weight tile by one activation vector
// with mma.sync.m16n8k16 (f16 in, f32 accumulate).  Weights are the A
// operand, dequantised in registers straight from the raw GGUF bytes the
// TMA engine staged in shared memory; the activation vector is the B
// operand, split into an f16 high part and an f16 residual so that x is
// carried to ~22 bits (x_hi + x_lo), well inside the fp32-accumulate budget.
//
// Fragment layout of m16n8k16 (lane = 4*g + t): A rows g and g+8 at k-slots
// {2t, 2t+1, 2t+8, 2t+9}; B column g at the same k-slots; C row g / g+8 at
// columns 2t, 2t+1.  The k order inside a step is free as long as A and B
// agree, so every format chooses the order that keeps a thread's weights in
// one aligned 32-bit word: k-slots (2t, 2t+1, 2t+8, 2t+9) <- bytes
// (0, 2, 1, 3) of that word ("kPerm").
//
// "Column trick": B column 2t holds x_hi and column 2t+1 holds x_lo only at
// thread t's own k-slots (zero elsewhere), so after a run of steps lane
// (g, t) holds in C[2t] + C[2t+1] the dot product over exactly the weights
// thread t supplied.  Each thread can therefore follow its own scale group
// (Q8_0 block, Q6_K 16-value group) and apply that scale in fp32.
//
// Integer-valued dequantisation is exact in f16: 0x6400 | u is 1024 + u, so
// a byte or nibble placed in the low mantissa bits and a subtraction (or an
// FMA whose exact result is an integer below 2048) recovers the quant value
// (or scale * quant for Q4_K, whose 6-bit scale times 4-bit quant is < 2048).
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

constexpr int kSegElems = 256;  // every fast-path format works in 256-value segments
constexpr int kStepBytesB = 64; // B table bytes per k16 step: [t][hi,lo][4 x f16]
VHD int kperm(int j) { return (j == 0) ? 0 : (j == 1) ? 2 : (j == 2) ? 1 : 3; }

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
// segment, a 4-byte-aligned span of 17 words W0..W16:
//   W0 = [dA, dA, q0, q1], W1..W7 = q2..q29, W8 = [q30, q31, dB, dB],
//   W9..W16 = block B's 32 quants.
// Steps 0..6 use W1..W7, step 7 uses [q0,q1,q30,q31] = prmt(W0, W8), steps
// 8..15 use W9..W16.  After step 7 and step 15 the block's d scales C.
struct Q8 {
  static constexpr uint32_t kType = T_Q8_0;
  static constexpr int kSegBytes = 272, kSteps = 16;
  static constexpr int kSumGroup = 32;  // x sums per block (offset correction)
  VHD static int elem(int step, int t, int j) {
    int base = 64 * t;
    if (step < 7) return base + 2 + 4 * step + kperm(j);
    if (step == 7) return base + ((j == 0) ? 0 : (j == 1) ? 30 : (j == 2) ? 1 : 31);
    return base + 32 + 4 * (step - 8) + kperm(j);
  }
  // int8 x4 -> (f16x2 of bytes 0,2 ; f16x2 of bytes 1,3) holding 1152 + q,
  // exact.  One lop3 per pair: the sign bit of each byte is flipped (q+128
  // as an unsigned byte), the other byte of each half becomes 0x64; bit
  // classes per (b, c): (0,0) keep, (1,0) flip, (1,1) one, (0,1) zero.
  VHD static void conv(uint32_t w, uint32_t& h02, uint32_t& h13) {
    h02 = lop3t<0x9C>(w, 0x64806480u, 0xFF00FF00u);
    h13 = lop3t<0x9C>(w >> 8, 0x64806480u, 0xFF00FF00u);
  }
  static constexpr float kOffset = 1152.f;  // removed with the block sum of x
};

// ---- Q4_K: 144-byte super-blocks, segment = 1 super-block ---------------
// Thread t owns the 64-value chunk t: bytes qs[32t, 32t+32) (two 16-byte
// aligned loads); low nibbles are sub-block 2t, high nibbles sub-block
// 2t+1.  Step 2i uses the low nibbles of word i, step 2i+1 the high ones.
// The 6-bit sub-block scale is folded into A (sc*q <= 945, exact in f16);
// the super-block d and the min term -dmin*m_j*sum(x over sub-block j) are
// applied in fp32 once per segment.
struct Q4K {
  static constexpr uint32_t kType = T_Q4_K;
  static constexpr int kSegBytes = 144, kSteps = 16;
  static constexpr int kSumGroup = 32;  // x sums per sub-block (min term)
  VHD static int elem(int step, int t, int j) { return 64 * t + 32 * (step & 1) + 4 * (step >> 1) + kperm(j); }
  // low nibbles: halves 1024 + q (bytes 0,2) and (bytes 1,3)
  VHD static void conv_lo(uint32_t w, uint32_t& h02, uint32_t& h13) {
    h02 = (w & 0x000F000Fu) | 0x64006400u;
    h13 = ((w >> 8) & 0x000F000Fu) | 0x64006400u;
  }
  // high nibbles: halves 1024 + 16*q
  VHD static void conv_hi(uint32_t w, uint32_t& h02, uint32_t& h13) {
    h02 = (w & 0x00F000F0u) | 0x64006400u;
    h13 = ((w >> 8) & 0x00F000F0u) | 0x64006400u;
  }
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
// Four macro-steps m (half h = m>>1, l0 = 16*(m&1)), four steps each.  In a
// macro-step thread t follows stream t of half h: values 128h + 32t + l0 +
// (0..15), whose low 4 bits are the low (t<2) or high (t>=2) nibble of
// ql[64h + 32*(t&1) + l] and whose top 2 bits are bits (2t, 2t+1) of
// qh[32h + l]; one int8 scale (index 8h + 2t + l0/16) covers all 16.
// Super-blocks are only 2-byte aligned in general (210 = 2 mod 4), so
// words are read with a funnel shift.
struct Q6K {
  static constexpr uint32_t kType = T_Q6_K;
  static constexpr int kSegBytes = 210, kSteps = 16;
  static constexpr int kSumGroup = 16;  // x sums per scale group (offset correction)
  VHD static int elem(int step, int t, int j) {
    int m = step >> 2, s = step & 3;
    return 128 * (m >> 1) + 32 * t + 16 * (m & 1) + 4 * s + kperm(j);
  }
  // 4 six-bit values of stream t from a ql word and a qh word
  VHD static uint32_t six(uint32_t ql, uint32_t qh, int t) {
    uint32_t lo = (ql >> (4u * (uint32_t)(t >> 1))) & 0x0F0F0F0Fu;
    uint32_t hi = ((qh >> (2u * (uint32_t)t)) & 0x03030303u) << 4;
    return lo | hi;
  }
  // halves 1024 + z (z = the 6-bit value); value = z - 32, so the offset
  // removed with the group sum of x is 1056
  VHD static void conv(uint32_t z, uint32_t& h02, uint32_t& h13) {
    h02 = (z & 0x00FF00FFu) | 0x64006400u;
    h13 = byte_perm(z, 0x64646464u, 0x4341u);
  }
  static constexpr float kOffset = 1056.f;
};

}  // namespace vireo
