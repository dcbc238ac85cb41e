// Batched (prefill) MoE FFN on the fifth-generation tensor cores.
//
// The reference runs moe_ffn once per token (vireo src/gguf_run.c:185-214);
// for a batch of T tokens this computes the same function for every token at
// once, as grouped GEMMs over the experts:
//
//   prep     xa[t]   = the token's hidden vector as f16, columns permuted within
//                      groups of 4 (0 2 1 3), then the 32-value group sums
//                      (the Q4_K min-term block)
//   router   logits  = xa . (R_hi + R_lo)^T (+ bias): a tcgen05 GEMM against
//                      the fp32 router split into two f16 halves, fp32
//                      accumulate; epilogue = softmax, top-k (the reference's
//                      strict-'>' scan, ties to the lower id), renorm, and a
//                      count per expert
//   scan     per-expert row ranges padded to 128, the table of 256-row tiles
//            (a range's last tile may hold one 128-row sub-tile)
//   place    every (token, slot) pair gets a row of its expert's range; the
//            token's xa row is copied there
//   gate/up  h = silu(X_e W_gate,e^T) * (X_e W_up,e^T) for every expert's rows
//            (tcgen05 GEMM, Q4_K weights dequantised to f16 in shared memory)
//   down     y = w_pair * (H_e W_down,e^T) (Q6_K weights, f16), rounded to
//            f16 into the pair's token-slot row of the return buffer
//   combine  x[t] += sum over slots of y(t, slot), in slot order, fp32
//
// GEMM kernel (prefill_gemm<MODE>): persistent, one CTA per SM, 16 warps:
// warp 0 allocates TMEM (512 columns: two 128 x 256 fp32 accumulators) and
// issues the TMA loads of the activation tiles (128-byte swizzle; 256 rows x
// 64 K for the expert GEMMs, 128 rows for the router); warp 1 issues the
// tcgen05.mma (M 128, N 256, K 16) from one thread; warps 4-11 write the
// weight tiles (256 rows x 64 K) into shared memory, dequantising GGUF
// blocks straight into the swizzled f16 layout (the router's weight tile
// comes by TMA instead); warps 12-15 are the epilogue, reading their 32 TMEM
// lanes with tcgen05.ld (the router's top-k runs on warps 4-15).  Rings of stages (full / empty mbarriers) connect
// loads, dequantisation and MMAs.  In the expert GEMMs a tile's two 128-row
// sub-tiles go to the two accumulators and share every converted weight
// stage: the dequantisation, which bounded these GEMMs when each converted
// tile fed one sub-tile, is spread over twice the MMAs (the tile's epilogue
// no longer overlaps the next tile's MMAs).  The router GEMM alternates the
// two accumulators between tiles so its epilogue overlaps the next tile.
// Every wait is bounded (kWaitLimitNs) and sets the status word.
//
// Precision: activations and dequantised weights are f16 (the bf16 input is
// exact in f16 for |x| in [2^-14, 65504]); a weight is round(scale * q) with
// one rounding (the half2 FMA (1024 + q) * a - 1024 a is exact before its
// final rounding); accumulation is fp32.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <type_traits>

#include "engine.cuh"
#include "moe_decode.cuh"
#include "pdl_launch.cuh"
#include "umma.cuh"
#include "vireo_internal.h"

namespace vireo {

constexpr int kPM = 128;   // activation rows per tile
constexpr int kPN = 256;   // weight rows per tile
constexpr int kPK = 64;    // K per stage
constexpr int kPThreads = 512;
constexpr int kDqWarp0 = 4, kDqWarps = 8, kEpiWarp0 = 12;
constexpr int kPWarps = kPThreads / 32;
constexpr int kPTopK = 8;  // prefill top-k limit (held in registers)
constexpr int kPMaxPeers = 8;  // expert-parallel ranks (one node)
constexpr uint32_t kPStageA = kPM * kPK * 2, kPStageB = kPN * kPK * 2;
// raw weight chunks of one stage (the repacked layouts, 256 rows each):
// gate/up 48 B per row (Q4_K header + the stage's 32 quant bytes), down 80 B
// per row (64 six-bit values as bytes z + 96, then 4 f16 scales d sc)
constexpr uint32_t kPRawGU = kPN * 48, kPRawDN = kPN * 80;

// Three rings per GEMM: activation tiles (TMA, freed by the MMA), raw weight
// chunks (bulk copy, freed by the dequant warps) and converted weight tiles
// (written by the dequant warps, freed by the MMA).  The first two run
// several stages ahead of the MMA so their latency is hidden; only a few
// 32 KB converted tiles need to be resident.
#ifndef VIREO_P_NA_GU
#define VIREO_P_NA_GU 2
#endif
#ifndef VIREO_P_NB_GU
#define VIREO_P_NB_GU 3
#endif
#ifndef VIREO_P_NR_GU
#define VIREO_P_NR_GU 4
#endif
#ifndef VIREO_P_NA_DN
#define VIREO_P_NA_DN 2
#endif
#ifndef VIREO_P_NB_DN
#define VIREO_P_NB_DN 2
#endif
#ifndef VIREO_P_NR_DN
#define VIREO_P_NR_DN 3
#endif
// The expert GEMMs (gate/up, down) take 256-row tiles: two 128-row
// sub-tiles in two TMEM accumulators share every converted weight stage, so
// each dequantised tile feeds twice the MMAs.  The router GEMM keeps 128-row
// tiles and double-buffered accumulators.
template <int MODE>
__host__ __device__ constexpr int psub() {
  return MODE == 0 ? 1 : 2;
}
template <int MODE>
struct PRing {
  // activation stages, converted weight stages, raw chunk stages
  static constexpr int NA = MODE == 2 ? VIREO_P_NA_DN : (MODE == 1 ? VIREO_P_NA_GU : 4);
  static constexpr int NB = MODE == 2 ? VIREO_P_NB_DN : (MODE == 1 ? VIREO_P_NB_GU : 3);
  static constexpr int NR = MODE == 1 ? VIREO_P_NR_GU : (MODE == 2 ? VIREO_P_NR_DN : 1);
  static constexpr uint32_t RB = MODE == 2 ? kPRawDN : kPRawGU;   // raw chunk bytes
  static constexpr uint32_t SA = psub<MODE>() * kPStageA;          // activation stage bytes
  static constexpr uint32_t OFF_B = NA * SA;
  static constexpr uint32_t OFF_R = OFF_B + NB * kPStageB;
  static constexpr uint32_t BYTES = OFF_R + (MODE == 0 ? 0u : NR * RB);
};
constexpr uint32_t cmax(uint32_t a, uint32_t b) { return a > b ? a : b; }
// the down GEMM's epilogue stages each warp's 32-row x 64-column f16 output
// block here (row stride 33 words) when its rows return to other ranks
constexpr uint32_t kPEpiStage = 4 * 32 * 33 * 4;
// the router's epilogue spills each tile's logits here ([128][129] floats)
// so that twelve warps share the softmax and top-k
constexpr uint32_t kPLogits = kPM * (128 + 1) * 4;
template <int MODE>
constexpr uint32_t psmem() {
  return 1024 + PRing<MODE>::BYTES + (MODE == 2 ? kPEpiStage : 0u) + (MODE == 0 ? kPLogits : 0u);
}
static_assert(psmem<0>() <= 227 * 1024 && psmem<1>() <= 227 * 1024 && psmem<2>() <= 227 * 1024,
              "prefill rings exceed the shared memory of one CTA");

enum PMode { P_ROUTER = 0, P_GATEUP = 1, P_DOWN = 2 };

struct PTile {
  int e, row0, nrows;
};

struct PrefillParams {
  int T, d, fe, ne, k, renorm;
  int Kx;       // columns of xa / Xg: d + the Q4_K min block
  int nk;       // K stages of this GEMM
  int n_ntiles;
  const int* n_mtiles;  // device (gate/up, down)
  const PTile* tiles;   // device
  const uint8_t* const* exp_tab;
  const uint8_t* pack;   // repacked weight chunks of this GEMM
  uint32_t rb_gu, rb_d;  // row bytes of gate/up (Q4_K, d) and down (Q6_K, fe) rows
  // router
  const float* bias;
  int32_t* ids;
  float* wts;
  int* counts;
  // gate/up
  __half* hg;  // [rows][fe], columns permuted as xa's
  // down
  const float* wrow;
  // row r's output, as f16, goes to rank ysrc[r] >> 24's buffer
  // ypeer[rank], row ysrc[r] & 0xFFFFFF: the token slot's row of the
  // caller's return buffer (its own on one GPU; on several, peer memory
  // written over NVLink while the next tile's MMAs run)
  const int* ysrc;
  __half* ypeer[kPMaxPeers];
  int remote;  // some ypeer is another GPU's memory
  int* err;
};

VHD int swap4(int j) { return (j & ~3) | ((j & 1) << 1) | ((j >> 1) & 1); }

VDEV uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
VDEV __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// ---- bounded waits sharing a CTA abort flag ---------------------------------
VDEV bool pwait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
  if (mbar_wait(bar, parity, abort)) return true;
  if (!*abort) {
    set_error(err, VIREO_ERR_TIMEOUT);
    *abort = 1;
  }
  return false;
}

// ---- Q4_K chunk row -> 64 f16 of one K stage (gate/up B tiles) -------------
// Stage kt (< d / 64) = chunk c = kt & 3 of super-block kt >> 2.  Positions
// 0..31 are the low nibbles of qs[32c ..], 32..63 the high nibbles, each
// group of 4 ordered (0 2 1 3), as xa's columns.  Value = round(d sc_j q);
// the -dmin m_j terms come from the min-block stages (minmat, by TMA).
struct Q4Raw {
  uint4 hd, qa, qb;  // super-block header, the stage's 32 quant bytes
};

VDEV void conv_q4k(const Q4Raw& R, int kt, uint8_t* tile, int r) {
  const int c = kt & 3;
  const float dd = h_lo(R.hd.x);
  uint32_t sc0, m0, sc1, m1;
  Q4K::scale_min(R.hd.y, R.hd.z, R.hd.w, 2 * c, sc0, m0);
  Q4K::scale_min(R.hd.y, R.hd.z, R.hd.w, 2 * c + 1, sc1, m1);
  const float a0f = dd * (float)sc0, a1f = dd * (float)sc1 * 0.0625f;  // high nibbles come as 16 q
  const uint32_t w[8] = {R.qa.x, R.qa.y, R.qa.z, R.qa.w, R.qb.x, R.qb.y, R.qb.z, R.qb.w};
  const bool fast = fabsf(a0f) < 32.f && fabsf(a1f) < 32.f;  // 1024 a exact in f16
  const __half2 A0 = __float2half2_rn(a0f), A1 = __float2half2_rn(a1f);
  const __half2 C0 = __hmul2(A0, __float2half2_rn(-1024.f)), C1 = __hmul2(A1, __float2half2_rn(-1024.f));
  const __half2 K1024 = __float2half2_rn(1024.f);
  uint8_t* rowt = tile + r * 128;
  const int sw = r & 7;
  if (fast) {
#pragma unroll
    for (int ch = 0; ch < 8; ch++) {
      const uint32_t msk = ch < 4 ? 0x000F000Fu : 0x00F000F0u;
      const __half2 A = ch < 4 ? A0 : A1, C = ch < 4 ? C0 : C1;
      const uint32_t w0 = w[2 * (ch & 3)], w1 = w[2 * (ch & 3) + 1];
      const uint32_t h0 = h2u(__hfma2(u2h((w0 & msk) | 0x64006400u), A, C));
      const uint32_t h1 = h2u(__hfma2(u2h(((w0 >> 8) & msk) | 0x64006400u), A, C));
      const uint32_t h2 = h2u(__hfma2(u2h((w1 & msk) | 0x64006400u), A, C));
      const uint32_t h3 = h2u(__hfma2(u2h(((w1 >> 8) & msk) | 0x64006400u), A, C));
      *reinterpret_cast<uint4*>(rowt + ((ch ^ sw) << 4)) = make_uint4(h0, h1, h2, h3);
    }
  } else {
#pragma unroll
    for (int ch = 0; ch < 8; ch++) {
      const uint32_t msk = ch < 4 ? 0x000F000Fu : 0x00F000F0u;
      const __half2 A = ch < 4 ? A0 : A1;
      const uint32_t w0 = w[2 * (ch & 3)], w1 = w[2 * (ch & 3) + 1];
      const uint32_t u[4] = {(w0 & msk) | 0x64006400u, ((w0 >> 8) & msk) | 0x64006400u, (w1 & msk) | 0x64006400u,
                             ((w1 >> 8) & msk) | 0x64006400u};
      uint32_t h[4];
#pragma unroll
      for (int i = 0; i < 4; i++) h[i] = h2u(__hmul2(__hsub2(u2h(u[i]), K1024), A));
      *reinterpret_cast<uint4*>(rowt + ((ch ^ sw) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
}

// ---- repacked Q6_K chunk row (shared memory) -> 64 f16 of one stage --------
// bytes 0..63: z + 96 of the stage's 64 values in natural order (z the 6-bit
// quant); bytes 64..71: f16 d sc of the four 16-value groups.  Value =
// ((1024 + z + 96) - 1152) * d sc, the subtraction exact.
VDEV void conv_dn(const uint8_t* raw, uint8_t* tile, int r) {
  const uint4 v0 = *reinterpret_cast<const uint4*>(raw), v1 = *reinterpret_cast<const uint4*>(raw + 16);
  const uint4 v2 = *reinterpret_cast<const uint4*>(raw + 32), v3 = *reinterpret_cast<const uint4*>(raw + 48);
  const uint2 sc = *reinterpret_cast<const uint2*>(raw + 64);
  const uint32_t w[16] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w, v2.x, v2.y, v2.z, v2.w, v3.x, v3.y, v3.z, v3.w};
  const __half2 K1152 = __float2half2_rn(1152.f);
  uint8_t* rowt = tile + r * 128;
  const int sw = r & 7;
#pragma unroll
  for (int ch = 0; ch < 8; ch++) {
    const uint32_t sw2 = (ch >> 1) < 2 ? sc.x : sc.y;
    const uint32_t a16 = ((ch >> 1) & 1) ? (sw2 >> 16) : (sw2 & 0xFFFFu);
    const __half2 A = u2h(a16 | (a16 << 16));
    const uint32_t w0 = w[2 * ch], w1 = w[2 * ch + 1];
    const uint32_t h0 = h2u(__hmul2(__hsub2(u2h((w0 & 0x00FF00FFu) | 0x64006400u), K1152), A));
    const uint32_t h1 = h2u(__hmul2(__hsub2(u2h(((w0 >> 8) & 0x00FF00FFu) | 0x64006400u), K1152), A));
    const uint32_t h2 = h2u(__hmul2(__hsub2(u2h((w1 & 0x00FF00FFu) | 0x64006400u), K1152), A));
    const uint32_t h3 = h2u(__hmul2(__hsub2(u2h(((w1 >> 8) & 0x00FF00FFu) | 0x64006400u), K1152), A));
    *reinterpret_cast<uint4*>(rowt + ((ch ^ sw) << 4)) = make_uint4(h0, h1, h2, h3);
  }
}

template <int MODE>
__global__ void __launch_bounds__(kPThreads, 1)
    prefill_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ PrefillParams p) {
  pdl_wait();  // launched with programmatic serialization: the previous kernel is complete
  extern __shared__ __align__(1024) uint8_t praw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)praw + 1023) & ~(uintptr_t)1023);
  using RG = PRing<MODE>;
  constexpr int NA = RG::NA, NB = RG::NB, NR = RG::NR;
  uint8_t* sA = sm;
  uint8_t* sB = sm + RG::OFF_B;
  uint8_t* sR = sm + RG::OFF_R;
  __shared__ uint64_t fullA[NA], emptyA[NA], fullB[NB], emptyB[NB], rawfull[NR], rawempty[NR];
  __shared__ uint64_t tfull[2], tempty[2], drain;
  __shared__ uint32_t tbase;
  __shared__ int n_items_s;
  __shared__ volatile int abort_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NA; i++) {
      mbar_init(&fullA[i], 1);
      mbar_init(&emptyA[i], 1);
    }
    for (int i = 0; i < NB; i++) {
      mbar_init(&fullB[i], MODE == P_ROUTER ? 1u : (uint32_t)kDqWarps);
      mbar_init(&emptyB[i], 1);
    }
    for (int i = 0; i < NR; i++) {
      mbar_init(&rawfull[i], 1);
      mbar_init(&rawempty[i], kDqWarps);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(&drain, 1);
    mbar_fence_init();
    abort_s = 0;
    // router: n_ntiles CTAs per row tile, each selecting for its share of the rows
    n_items_s = MODE == P_ROUTER ? (p.T + kPM - 1) / kPM * p.n_ntiles : (*p.n_mtiles) * p.n_ntiles;
  }
  if (warp == 0) tmem_alloc(&tbase, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tbase;
  const int n_items = n_items_s;
  const int nkd = MODE == P_GATEUP ? p.d / kPK : p.nk;  // stages with a raw chunk (all but the min block)
  auto tile_of = [&](int mt) -> PTile {
    if constexpr (MODE == P_ROUTER) {
      PTile t;
      t.e = 0;
      t.row0 = mt * kPM;
      t.nrows = min(kPM, p.T - mt * kPM);
      return t;
    } else {
      return p.tiles[mt];
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer: activation tiles (TMA; the router's weight tiles too) ---
      uint32_t g = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items && !abort_s; item += gridDim.x) {
        const PTile t = tile_of(item / p.n_ntiles);
        for (int kt = 0; kt < p.nk; kt++, g++) {
          // every wait of the stage comes before any of its copies is issued,
          // so an abort leaves no copy untracked by the drain below
          const int a = (int)(g % NA), b = (int)(g % NB);
          if ((g >= (uint32_t)NA && !pwait(&emptyA[a], ((g / NA) - 1) & 1, &abort_s, p.err)) ||
              (MODE == P_ROUTER && g >= (uint32_t)NB && !pwait(&emptyB[b], ((g / NB) - 1) & 1, &abort_s, p.err))) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&fullA[a], RG::SA);
          tma_load_2d(sA + a * RG::SA, &tmA, kt * kPK, t.row0, &fullA[a]);
          if constexpr (MODE == P_ROUTER) {
            mbar_arrive_expect_tx(&fullB[b], kPStageB);
            tma_load_2d(sB + b * kPStageB, &tmB, kt * kPK, 0, &fullB[b]);
          }
        }
      }
      // the copies this thread issued land before the CTA may exit
      volatile int never = 0;
      for (uint32_t j = g > (uint32_t)NA ? g - NA : 0; j < g; j++) mbar_wait(&fullA[j % NA], (j / NA) & 1, &never);
      if (MODE == P_ROUTER)
        for (uint32_t j = g > (uint32_t)NB ? g - NB : 0; j < g; j++) mbar_wait(&fullB[j % NB], (j / NB) & 1, &never);
    }
  } else if (warp == 2) {
    if constexpr (MODE != P_ROUTER) {
      if (lane == 0) {
        // ---- producer: raw weight chunks (bulk copies), paced only by the
        // dequantisation warps, so the chunk ring runs ahead of the MMAs -----
        uint32_t rg = 0;
        bool ok = true;
        for (int item = blockIdx.x; ok && item < n_items && !abort_s; item += gridDim.x) {
          const PTile t = tile_of(item / p.n_ntiles);
          const int nt = item % p.n_ntiles;
          for (int kt = 0; kt < nkd; kt++, rg++) {
            const int sl = (int)(rg % NR);
            if (rg >= (uint32_t)NR && !pwait(&rawempty[sl], ((rg / NR) - 1) & 1, &abort_s, p.err)) {
              ok = false;
              break;
            }
            const uint8_t* src = p.pack + ((size_t)(t.e * p.n_ntiles + nt) * nkd + kt) * RG::RB;
            mbar_arrive_expect_tx(&rawfull[sl], RG::RB);
            bulk_g2s(sR + sl * RG::RB, src, RG::RB, &rawfull[sl]);
          }
        }
        volatile int never = 0;
        for (uint32_t j = rg > (uint32_t)NR ? rg - NR : 0; j < rg; j++)
          mbar_wait(&rawfull[j % NR], (j / NR) & 1, &never);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer --------------------------------------------------------
      constexpr uint32_t idesc = umma_idesc_f16(kPM, kPN);
      uint32_t g = 0;
      int it = 0;
      for (int item = blockIdx.x; item < n_items && !abort_s; item += gridDim.x, it++) {
        // router: two 256-column accumulators, alternating (the epilogue of
        // one tile overlaps the next tile's MMAs); expert GEMMs: one pair of
        // accumulators, sub-tile s in columns 256 s .. 256 s + 255
        const int b2 = MODE == P_ROUTER ? (it & 1) : 0;
        if constexpr (MODE == P_ROUTER) {
          if (it >= 2 && !pwait(&tempty[b2], ((it >> 1) - 1) & 1, &abort_s, p.err)) break;
        } else {
          if (it >= 1 && !pwait(&tempty[0], (it - 1) & 1, &abort_s, p.err)) break;
        }
        tc_fence_after();
        const uint32_t dt = tmem + (uint32_t)(b2 * kPN);
        // the second sub-tile only when the tile has rows there
        const bool two = MODE != P_ROUTER && tile_of(item / p.n_ntiles).nrows > kPM;
        bool ok = true;
        for (int kt = 0; kt < p.nk; kt++, g++) {
          const int a = (int)(g % NA), b = (int)(g % NB);
          if (!pwait(&fullA[a], (g / NA) & 1, &abort_s, p.err) || !pwait(&fullB[b], (g / NB) & 1, &abort_s, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(sA + a * RG::SA), db = umma_desc_sw128(sB + b * kPStageB);
#pragma unroll
          for (int kk = 0; kk < kPK / 16; kk++)
            umma_f16_ss(dt, da + 2 * kk, db + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
          if (two) {
            const uint64_t da1 = umma_desc_sw128(sA + a * RG::SA + kPStageA);
#pragma unroll
            for (int kk = 0; kk < kPK / 16; kk++)
              umma_f16_ss(dt + (uint32_t)kPN, da1 + 2 * kk, db + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&emptyA[a]);
          umma_commit(&emptyB[b]);
        }
        if (!ok) break;
        umma_commit(&tfull[b2]);
      }
      // every MMA issued here is complete before TMEM may be released
      umma_commit(&drain);
      volatile int never = 0;
      mbar_wait(&drain, 0, &never);
    }
  } else if (MODE == P_ROUTER && warp >= kDqWarp0) {
    if constexpr (MODE == P_ROUTER) {
      // ---- router epilogue: logits = hi + lo (+ bias); softmax; top-k; renorm
      // (gguf_run.c:187-192).  The four epilogue warps move each row's logits
      // from TMEM to shared memory and free the accumulator; then the twelve
      // warps 4-15 (the dequantisation warps have no weights to convert here)
      // take the rows, eight lanes per row, sixteen experts per lane: the
      // max and the sum by a 3-step xor tree, each lane's top k of its
      // experts by the reference's rule (strict '>' in increasing id, so the
      // lower id stays ahead of an equal one; NaN never enters), then k
      // rounds that take the best head among the eight lanes under (value
      // desc, id asc).  Slots beyond the valid experts hold id -1, weight -1.
      float* lgs = reinterpret_cast<float*>(sm + RG::BYTES);
      constexpr int kSelThreads = 32 * (kPWarps - kDqWarp0), kGroups = kSelThreads / 8;
      static_assert(kGroups % 4 == 0, "a warp's four row groups stay together across iterations");
      const int st = threadIdx.x - 32 * kDqWarp0, grp = st >> 3, j = st & 7;
      const int ne = p.ne, k = p.k;
      int it = 0;
      const int rpp = kPM / p.n_ntiles;  // rows per part (a multiple of 4)
      for (int item = blockIdx.x; item < n_items; item += gridDim.x, it++) {
        const PTile t = tile_of(item / p.n_ntiles);
        const int rb = (item % p.n_ntiles) * rpp, nsel = min(t.nrows, rb + rpp) - rb;
        if (warp >= kEpiWarp0) {
          const int q = warp & 3, b = it & 1;
          int w_ok = 0;
          if (!__any_sync(0xffffffffu, abort_s != 0)) {
            if (lane == 0) w_ok = pwait(&tfull[b], (it >> 1) & 1, &abort_s, p.err);
            w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
          }
          if (w_ok) {
            if (32 * q < rb + rpp && 32 * q + 32 > rb) {  // this warp's 32 rows meet the part's
              tc_fence_after();
              const int rt = 32 * q + lane;
              const uint32_t ta = tmem + (uint32_t)(b * kPN) + ((uint32_t)(32 * q) << 16);
              for (int c = 0; c < 128; c += 32) {
                uint32_t vh[32], vl[32];
                tmem_ld32(ta + c, vh);
                tmem_ld32(ta + 128 + c, vl);
#pragma unroll
                for (int jj = 0; jj < 32; jj++) {
                  const int e = c + jj;
                  lgs[rt * 129 + e] = e < ne ? __uint_as_float(vh[jj]) + __uint_as_float(vl[jj]) + (p.bias ? p.bias[e] : 0.f)
                                             : -INFINITY;
                }
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
          }
        }
        asm volatile("bar.sync 5, %0;" ::"r"(kSelThreads) : "memory");  // the tile's logits are in shared memory
        if (!__any_sync(0xffffffffu, abort_s != 0)) {
          // a warp takes four rows at a time, so all its lanes run the same
          // iterations (the shuffles name the whole warp); lanes past the
          // tile's last row compute on rows the logit buffer holds and write
          // nothing
          for (int rr = grp; (rr & ~3) < nsel; rr += kGroups) {
            const int r = rb + rr;
            const float* L = lgs + r * 129 + 16 * j;
            float ex[16];
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < 16; i++) {
              ex[i] = L[i];
              mx = fmaxf(mx, ex[i]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) {
              ex[i] = 16 * j + i < ne ? expf(ex[i] - mx) : 0.f;
              sum += ex[i];
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            float tv[kPTopK];
            int ti[kPTopK];
#pragma unroll
            for (int i = 0; i < kPTopK; i++) {
              tv[i] = -1.f;
              ti[i] = -1;
            }
#pragma unroll
            for (int i = 0; i < 16; i++) {
              const int e = 16 * j + i;
              if (e >= ne) continue;
              float pe = ex[i] / sum;  // NaN never enters (strict '>')
              int pe_i = e;
              // insert before the first strictly smaller entry; everything
              // after it shifts down one slot (an entry equal to its new
              // neighbour keeps its place ahead of it: it has the lower id)
              bool moved = false;
#pragma unroll
              for (int u = 0; u < kPTopK; u++) {
                if (u < k && (moved || pe > tv[u])) {
                  moved = true;
                  const float fv = tv[u];
                  const int fi = ti[u];
                  tv[u] = pe;
                  ti[u] = pe_i;
                  pe = fv;
                  pe_i = fi;
                }
              }
            }
            float ov[kPTopK];
            int oi[kPTopK];
#pragma unroll
            for (int u = 0; u < kPTopK; u++) {
              float bv = tv[0];
              int bi = ti[0];
#pragma unroll
              for (int o = 1; o < 8; o <<= 1) {
                const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
                const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
                // (value desc, id asc); an empty head (-1) loses to any expert
                if (i2 >= 0 && (bi < 0 || v2 > bv || (v2 == bv && i2 < bi))) {
                  bv = v2;
                  bi = i2;
                }
              }
              ov[u] = bv;
              oi[u] = bi;
              if (bi >= 0 && ti[0] == bi) {  // the lane that held it moves to its next
#pragma unroll
                for (int w2 = 0; w2 < kPTopK - 1; w2++) {
                  tv[w2] = tv[w2 + 1];
                  ti[w2] = ti[w2 + 1];
                }
                tv[kPTopK - 1] = -1.f;
                ti[kPTopK - 1] = -1;
              }
            }
            if (j == 0 && rr < nsel) {
              float ws = 0.f;
#pragma unroll
              for (int u = 0; u < kPTopK; u++)
                if (u < k) ws = ws + (oi[u] >= 0 ? ov[u] : -1.f);
              const int row = t.row0 + r;
#pragma unroll
              for (int u = 0; u < kPTopK; u++) {
                if (u < k) {
                  const float v = oi[u] >= 0 ? ov[u] : -1.f;
                  const float w = (p.renorm && ws > 0.f) ? v / ws : v;
                  p.ids[(size_t)row * k + u] = oi[u];
                  p.wts[(size_t)row * k + u] = w;
                  if (oi[u] >= 0) atomicAdd(&p.counts[oi[u]], 1);
                }
              }
            }
          }
        }
        asm volatile("bar.sync 5, %0;" ::"r"(kSelThreads) : "memory");  // the logit buffer is free for the next tile
      }
    }
  } else if (warp >= kDqWarp0 && warp < kDqWarp0 + kDqWarps) {
    if constexpr (MODE != P_ROUTER) {
      // ---- weight tiles: raw chunks -> swizzled f16 in shared memory ----------
      // Each thread owns one tile row: it waits for the stage's converted-tile
      // slot to be free (emptyB) and its raw chunk to land (rawfull), converts
      // its row, frees the raw slot (rawempty) and the warp arrives on fullB.
      // A gate/up min-block stage is loaded into the slot by TMA instead (one
      // lane of the first dequant warp; its arrive.expect_tx is that warp's
      // arrival).
      const int r = threadIdx.x - 32 * kDqWarp0;  // tile row 0..255
      uint32_t g = 0, rg = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items && !abort_s; item += gridDim.x) {
        const PTile t = tile_of(item / p.n_ntiles);
        const int nt = item % p.n_ntiles;
        for (int kt = 0; kt < p.nk; kt++, g++) {
          const int b = (int)(g % NB);
          int w_ok = 1;
          if (lane == 0 && g >= (uint32_t)NB) w_ok = pwait(&emptyB[b], ((g / NB) - 1) & 1, &abort_s, p.err);
          const bool is_raw = kt < nkd;
          const int sl = (int)(rg % NR);
          if (lane == 0 && w_ok && is_raw) w_ok = pwait(&rawfull[sl], (rg / NR) & 1, &abort_s, p.err);
          w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
          if (!w_ok) {
            ok = false;
            break;
          }
          uint8_t* tile = sB + b * kPStageB;
          if (is_raw) {
            if constexpr (MODE == P_GATEUP) {
              const uint8_t* raw = sR + sl * RG::RB + r * 48;
              Q4Raw q;
              q.hd = *reinterpret_cast<const uint4*>(raw);
              q.qa = *reinterpret_cast<const uint4*>(raw + 16);
              q.qb = *reinterpret_cast<const uint4*>(raw + 32);
              conv_q4k(q, kt, tile, r);
            } else {
              conv_dn(sR + sl * RG::RB + r * 80, tile, r);
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              mbar_arrive(&rawempty[sl]);
              mbar_arrive(&fullB[b]);
            }
            rg++;
          } else if constexpr (MODE == P_GATEUP) {
            if (lane == 0) {
              if (warp == kDqWarp0) {
                const int y0 = t.e * 2 * p.fe + nt * 128, x0 = (kt - nkd) * kPK;
                mbar_arrive_expect_tx(&fullB[b], kPStageB);
                tma_load_2d(tile, &tmB, x0, y0, &fullB[b]);
                tma_load_2d(tile + kPStageB / 2, &tmB, x0, y0 + p.fe, &fullB[b]);
              } else {
                mbar_arrive(&fullB[b]);
              }
            }
          }
        }
      }
      // a min-block load issued here lands before the CTA may exit (stage j
      // of this loop is stage j % nk of its tile)
      if (warp == kDqWarp0 && lane == 0 && MODE == P_GATEUP) {
        volatile int never = 0;
        for (uint32_t j = g > (uint32_t)NB ? g - NB : 0; j < g; j++)
          if ((int)(j % (uint32_t)p.nk) >= nkd) mbar_wait(&fullB[j % NB], (j / NB) & 1, &never);
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ---- epilogue ------------------------------------------------------------
    const int q = warp & 3;
    int it = 0;
    for (int item = blockIdx.x; item < n_items && !abort_s; item += gridDim.x, it++) {
      const int b = MODE == P_ROUTER ? (it & 1) : 0;
      int w_ok = 1;
      if (lane == 0) w_ok = pwait(&tfull[b], MODE == P_ROUTER ? (it >> 1) & 1 : it & 1, &abort_s, p.err);
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      if (!w_ok) break;
      tc_fence_after();
      const int mt = item / p.n_ntiles, nt = item - mt * p.n_ntiles;
      const PTile t = tile_of(mt);
      for (int sub = 0; sub < psub<MODE>(); sub++) {
      if (sub > 0 && t.nrows <= kPM) break;  // no rows in the second sub-tile
      const int rt = kPM * sub + 32 * q + lane;  // row within the tile
      const bool valid = rt < t.nrows;
      const int row = t.row0 + rt;
      const uint32_t ta = tmem + (uint32_t)((b + sub) * kPN) + ((uint32_t)(32 * q) << 16);
      if constexpr (MODE == P_GATEUP) {
        // h = silu(g) * u (gguf_run.c:206), f16, columns permuted as xa's
        const int f0 = nt * 128;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t vg[32], vu[32];
          tmem_ld32(ta + c, vg);
          tmem_ld32(ta + 128 + c, vu);
          uint32_t hp[16];
#pragma unroll
          for (int j4 = 0; j4 < 8; j4++) {
            float hv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const float g = __uint_as_float(vg[4 * j4 + i]), u = __uint_as_float(vu[4 * j4 + i]);
              // fast exp and divide: h is rounded to f16 (2^-11) right after
              hv[i] = __fdividef(g, 1.0f + __expf(-g)) * u;
            }
            // positions (0 2 1 3) within the group of 4
            hp[2 * j4] = h2u(__floats2half2_rn(hv[0], hv[2]));
            hp[2 * j4 + 1] = h2u(__floats2half2_rn(hv[1], hv[3]));
          }
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(p.hg + (size_t)row * p.fe + f0 + c);
#pragma unroll
            for (int i = 0; i < 4; i++) dst[i] = make_uint4(hp[4 * i], hp[4 * i + 1], hp[4 * i + 2], hp[4 * i + 3]);
          }
        }
      } else {
        // y = w * (H W_down^T), rounded to f16 into its token slot's row of
        // the return buffer (on several GPUs, the source rank's; half the
        // bytes of fp32, on NVLink and in the combine).  A thread holds one
        // row, so the warp's 32 rows are staged per 64-column chunk in shared
        // memory and stored row by row, 8 lanes per row: every store is a
        // whole 128-byte line.
        const int n0 = nt * kPN;
        const float w = valid ? p.wrow[row] : 0.f;
        {
          uint32_t* stg = reinterpret_cast<uint32_t*>(sm + RG::BYTES) + q * (32 * 33);
          unsigned long long dst = 0;
          if (valid) {
            const int src = p.ysrc[row];
            dst = reinterpret_cast<unsigned long long>(p.ypeer[src >> 24] + (size_t)(src & 0xFFFFFF) * p.d + n0);
          }
#pragma unroll 1
          for (int c = 0; c < kPN; c += 64) {
            uint32_t v0[32], v1[32];
            tmem_ld32(ta + c, v0);
            tmem_ld32(ta + c + 32, v1);
#pragma unroll
            for (int j = 0; j < 16; j++) {
              stg[lane * 33 + j] =
                  h2u(__floats2half2_rn(__uint_as_float(v0[2 * j]) * w, __uint_as_float(v0[2 * j + 1]) * w));
              stg[lane * 33 + 16 + j] =
                  h2u(__floats2half2_rn(__uint_as_float(v1[2 * j]) * w, __uint_as_float(v1[2 * j + 1]) * w));
            }
            __syncwarp();
#pragma unroll
            for (int pass = 0; pass < 8; pass++) {
              const int rr = 4 * pass + (lane >> 3), c8 = lane & 7;
              const unsigned long long drow = __shfl_sync(0xffffffffu, dst, rr);
              if (drow) {
                const uint32_t* sr = stg + rr * 33 + 4 * c8;
                reinterpret_cast<uint4*>(drow)[(c >> 3) + c8] = make_uint4(sr[0], sr[1], sr[2], sr[3]);
              }
            }
            __syncwarp();
          }
        }
      }
      }  // sub-tiles
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }
  if (MODE == P_DOWN && p.remote) __threadfence_system();  // peer rows written before the kernel ends
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---- prep: xa[t] = [f16 of the token's values, columns (0 2 1 3) per group
// of 4 | f16 of the 32-value group sums | zero padding], Kx columns --------
__global__ void prefill_prep(const __nv_bfloat16* hb, __half* xa, int T, int d, int Kx, int* counts) {
  pdl_wait();
  const int t = blockIdx.x;
  // the router's per-expert counts start at zero (in place of a memset, which
  // would break the chain of dependent launches)
  if (t == 0 && threadIdx.x < 256) counts[threadIdx.x] = 0;
  if (t >= T) return;
  const __nv_bfloat16* src = hb + (size_t)t * d;
  __half* dst = xa + (size_t)t * Kx;
  for (int j0 = 8 * threadIdx.x; j0 < d; j0 += 8 * blockDim.x) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __half2float(__float2half_rn(__bfloat162float(src[j0 + i])));
    uint32_t o[4];
    // positions j0 + (0 1 2 3) hold natural (0 2 1 3)
    o[0] = h2u(__floats2half2_rn(v[0], v[2]));
    o[1] = h2u(__floats2half2_rn(v[1], v[3]));
    o[2] = h2u(__floats2half2_rn(v[4], v[6]));
    o[3] = h2u(__floats2half2_rn(v[5], v[7]));
    *reinterpret_cast<uint4*>(dst + j0) = make_uint4(o[0], o[1], o[2], o[3]);
    // group sum of 32 values = 4 consecutive threads' 8 values
    float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((threadIdx.x & 3) == 0) dst[d + j0 / 32] = __float2half_rn(s);
  }
  for (int j = d + d / 32 + threadIdx.x; j < Kx; j += blockDim.x) dst[j] = __float2half_rn(0.f);
}

// ---- router weights as f16 hi/lo rows (256 x d), columns as xa's ----------
__global__ void prefill_router_split(const float* R, __half* R2, int ne, int d) {
  const int row = blockIdx.x;  // 0..255
  const int e = row & 127;
  const bool lo = row >= 128;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float v = 0.f;
    if (e < ne) {
      const float r = R[(size_t)e * d + swap4(j)];
      const float rh = __half2float(__float2half_rn(r));
      v = lo ? r - rh : r;
    }
    R2[(size_t)row * d + j] = __float2half_rn(v);
  }
}

// ---- Q4_K min block: minmat[e * 2fe + row][j] = -round(dmin m_j) of
// sub-block j of gate row (row < fe) or up row (row - fe) of expert e;
// columns d/32 .. Km zero ----------------------------------------------------
__global__ void prefill_minmat(const uint8_t* const* exp_tab, const int* own, int d, int fe, int Km, uint32_t rb,
                               __half* out) {
  const int row = blockIdx.x, e = row / (2 * fe), rr = row - e * 2 * fe;
  if (own && !own[e]) return;  // expert held by another rank: its bytes are never read
  const uint8_t* rowp = exp_tab[3 * e + (rr < fe ? 0 : 1)] + (size_t)(rr < fe ? rr : rr - fe) * rb;
  for (int j = threadIdx.x; j < Km; j += blockDim.x) {
    float v = 0.f;
    if (j < d / 32) {
      const uint32_t* hp = reinterpret_cast<const uint32_t*>(rowp + (j >> 3) * 144);
      uint32_t sc, mn;
      Q4K::scale_min(__ldg(hp + 1), __ldg(hp + 2), __ldg(hp + 3), j & 7, sc, mn);
      v = -(h_hi(__ldg(hp)) * (float)mn);
    }
    out[(size_t)row * Km + j] = __float2half_rn(v);
  }
}

// ---- repacking (once per layer): the raw bytes of each (expert, n-tile,
// stage) in one contiguous chunk, rows in tile order -------------------------
// gate/up: chunk (e * fe/128 + nt) * d/64 + kt, row r < 128 gate row nt 128 + r,
// r >= 128 up row nt 128 + r - 128: the Q4_K header and quant bytes 32c.. of
// super-block kt / 4 (c = kt % 4)
__global__ void prefill_pack_gu(const uint8_t* const* exp_tab, const int* own, int d, int fe, uint32_t rb,
                                uint8_t* out) {
  const int nkd = d / kPK, ntl = fe / 128;
  const int b = blockIdx.x, kt = b % nkd, ent = b / nkd, nt = ent % ntl, e = ent / ntl, r = threadIdx.x;
  if (own && !own[e]) return;
  const uint8_t* sbp =
      exp_tab[3 * e + (r < 128 ? 0 : 1)] + (size_t)(nt * 128 + (r & 127)) * rb + (size_t)(kt >> 2) * 144;
  const int c = kt & 3;
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)b * kPRawGU + r * 48);
  dst[0] = __ldg(reinterpret_cast<const uint4*>(sbp));
  dst[1] = __ldg(reinterpret_cast<const uint4*>(sbp + 16 + 32 * c));
  dst[2] = __ldg(reinterpret_cast<const uint4*>(sbp + 32 + 32 * c));
}

// down: chunk (e * d/256 + nt) * fe/64 + kt, row r = down row nt 256 + r: the
// stage's 64 values (quarter q = kt % 4 of super-block kt / 4: streams
// 2 (q & 1) and 2 (q & 1) + 1 of half q / 2, vireo gguf_compute.c:88-99) as
// bytes z + 96 in natural order, then f16 d sc of the four 16-value groups
__global__ void prefill_pack_dn(const uint8_t* const* exp_tab, const int* own, int d, int fe, uint32_t rb,
                                uint8_t* out) {
  const int nkf = fe / kPK, ntl = d / kPN;
  const int b = blockIdx.x, kt = b % nkf, ent = b / nkf, nt = ent % ntl, e = ent / ntl, r = threadIdx.x;
  if (own && !own[e]) return;
  const uint8_t* sbp = exp_tab[3 * e + 2] + (size_t)(nt * kPN + r) * rb + (size_t)(kt >> 2) * 210;
  const int q = kt & 3, h = q >> 1, s0 = 2 * (q & 1);
  uint8_t* dst = out + (size_t)b * kPRawDN + r * 80;
  uint32_t words[16];
#pragma unroll
  for (int i = 0; i < 16; i++) {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int v = 4 * i + j, st = s0 + (v >> 5), l = v & 31;
      const uint32_t lo = (__ldg(sbp + 64 * h + 32 * (st & 1) + l) >> (4 * (st >> 1))) & 15u;
      const uint32_t hi = (__ldg(sbp + 128 + 32 * h + l) >> (2 * st)) & 3u;
      w |= ((lo | (hi << 4)) + 96u) << (8 * j);
    }
    words[i] = w;
  }
  const float dd = __half2float(__ushort_as_half((unsigned short)(__ldg(sbp + 208) | (__ldg(sbp + 209) << 8))));
  uint32_t scw[2];
#pragma unroll
  for (int g2 = 0; g2 < 2; g2++) {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int grp = 2 * g2 + j, st = s0 + (grp >> 1);
      const int8_t sc = (int8_t)__ldg(sbp + 192 + 8 * h + 2 * st + (grp & 1));
      w |= (uint32_t)__half_as_ushort(__float2half_rn(dd * (float)sc)) << (16 * j);
    }
    scw[g2] = w;
  }
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; i++) d4[i] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
  d4[4] = make_uint4(scw[0], scw[1], 0u, 0u);
}

// ---- scan: padded row ranges, the tile table, placement cursors ------------
__global__ void prefill_scan(const int* counts, int ne, int* cursor, PTile* tiles, int* n_mtiles) {
  pdl_wait();
  // ranges padded to kPM rows; tiles of up to 2 kPM rows (the expert GEMMs'
  // two sub-tiles), a range's last tile possibly one sub-tile
  constexpr int kT = 2 * kPM;
  __shared__ int mts[256], offs[256];
  const int e = threadIdx.x;
  const int n = e < ne ? counts[e] : 0;
  mts[e] = (n + kT - 1) / kT;
  offs[e] = (n + kPM - 1) / kPM * kPM;
  __syncthreads();
  if (e == 0) {
    int mt = 0, off = 0;
    for (int i = 0; i < ne; i++) {
      const int m = mts[i], pad = offs[i];
      mts[i] = mt;
      offs[i] = off;
      mt += m;
      off += pad;
    }
    *n_mtiles = mt;
  }
  __syncthreads();
  if (e < ne) {
    cursor[e] = offs[e];
    for (int i = 0; i * kT < n; i++) {
      PTile t;
      t.e = e;
      t.row0 = offs[e] + i * kT;
      t.nrows = min(kT, n - i * kT);
      tiles[mts[e] + i] = t;
    }
  }
}

// ---- place: a row per (token, slot), the token's xa row copied there; the
// row's return slot is the pair itself (rank 0) ---------------------------
__global__ void prefill_place(const int32_t* ids, const float* wts, const __half* __restrict__ xa, int T, int k,
                              int Kx, int* cursor, int* ysrc, float* wrow, __half* __restrict__ xg) {
  pdl_wait();
  const int pair = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pair >= T * k) return;
  int pos = -1;
  if (lane == 0) {
    const int e = ids[pair];
    if (e >= 0) {
      pos = atomicAdd(&cursor[e], 1);
      wrow[pos] = wts[pair];
      ysrc[pos] = pair;
    }
  }
  pos = __shfl_sync(0xffffffffu, pos, 0);
  if (pos < 0) return;
  const uint4* s = reinterpret_cast<const uint4*>(xa + (size_t)(pair / k) * Kx);
  uint4* dst = reinterpret_cast<uint4*>(xg + (size_t)pos * Kx);
  // a lane's loads of a chunk are all issued before its stores (one chunk
  // is a whole row up to d = 2240)
  constexpr int kPlaceVec = 9;
  const int n16 = Kx / 8;
  for (int c0 = lane; c0 < n16; c0 += 32 * kPlaceVec) {
    uint4 v[kPlaceVec];
#pragma unroll
    for (int j = 0; j < kPlaceVec; j++)
      if (c0 + 32 * j < n16) v[j] = __ldg(s + c0 + 32 * j);
#pragma unroll
    for (int j = 0; j < kPlaceVec; j++)
      if (c0 + 32 * j < n16) dst[c0 + 32 * j] = v[j];
  }
}

// ---- expand (expert-parallel owner): a token's row crosses NVLink once per
// owner, into the receive buffer; each of the owner's rows whose source slot
// xsrc[row] is set copies it from there (rows placed directly hold -1).
// gridDim.y blocks per M tile, a warp per row.
__global__ void prefill_expand(const PTile* tiles, const int* n_mtiles, const int* xsrc, const __half* __restrict__ xr,
                               __half* __restrict__ xg, int Kx, int n_slots) {
  pdl_wait();
  if ((int)blockIdx.x >= *n_mtiles) return;
  const PTile t = tiles[blockIdx.x];
  const int lane = threadIdx.x & 31, n16 = Kx / 8;
  constexpr int kVec = 9;
  for (int i = (threadIdx.x >> 5) + blockIdx.y * (blockDim.x / 32); i < t.nrows; i += gridDim.y * (blockDim.x / 32)) {
    const int row = t.row0 + i, src = xsrc[row];
    if (src < 0 || src >= n_slots) continue;
    const uint4* s4 = reinterpret_cast<const uint4*>(xr + (size_t)src * Kx);
    uint4* d4 = reinterpret_cast<uint4*>(xg + (size_t)row * Kx);
    for (int c0 = lane; c0 < n16; c0 += 32 * kVec) {
      uint4 v[kVec];
#pragma unroll
      for (int j = 0; j < kVec; j++)
        if (c0 + 32 * j < n16) v[j] = __ldcs(s4 + c0 + 32 * j);
#pragma unroll
      for (int j = 0; j < kVec; j++)
        if (c0 + 32 * j < n16) d4[c0 + 32 * j] = v[j];
    }
  }
}

void prefill_expand_launch(const PrefillScratch* S, size_t rows, const int* xsrc, const __half* xr, int Kx,
                           int n_slots, cudaStream_t st) {
  rows = std::max<size_t>(rows, kPM);
  pdl_launch(prefill_expand, dim3((unsigned)(rows / kPM + 1), 8), dim3(256), 0, st, (const PTile*)S->tiles,
             (const int*)S->n_mtiles, xsrc, xr, (__half*)S->xg, Kx, n_slots);
}

// ---- combine: x[t] += sum in slot order of the f16 rows yret[t * k + i]
// (gguf_run.c:209, 213: moe_acc summed over the selected experts in order,
// then added to x), in fp32; eight columns per thread, the slots' loads
// issued together.  A slot whose id is -1 has no row.
__global__ void prefill_combine(const int32_t* ids, const __half* yret, float* x, int T, int k, int d) {
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= T) return;
  bool on[kPTopK];
#pragma unroll
  for (int i = 0; i < kPTopK; i++) on[i] = i < k && ids[(size_t)t * k + i] >= 0;
  const int d8 = d / 8;
  const uint4* y8 = reinterpret_cast<const uint4*>(yret) + (size_t)t * k * d8;
  float4* x4 = reinterpret_cast<float4*>(x) + (size_t)t * (d / 4);
  for (int c = threadIdx.x; c < d8; c += blockDim.x) {
    uint4 v[kPTopK];
#pragma unroll
    for (int i = 0; i < kPTopK; i++)
      if (on[i]) v[i] = __ldcs(y8 + (size_t)i * d8 + c);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kPTopK; i++)
      if (on[i]) {
        const uint32_t w4[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int h = 0; h < 4; h++) {
          const float2 f = __half22float2(u2h(w4[h]));
          acc[2 * h] = __fadd_rn(acc[2 * h], f.x);
          acc[2 * h + 1] = __fadd_rn(acc[2 * h + 1], f.y);
        }
      }
#pragma unroll
    for (int h = 0; h < 2; h++) {
      float4 xv = x4[2 * c + h];
      xv.x = __fadd_rn(xv.x, acc[4 * h]);
      xv.y = __fadd_rn(xv.y, acc[4 * h + 1]);
      xv.z = __fadd_rn(xv.z, acc[4 * h + 2]);
      xv.w = __fadd_rn(xv.w, acc[4 * h + 3]);
      x4[2 * c + h] = xv;
    }
  }
}

void prefill_combine_launch(const int32_t* ids, const __half* yret, float* x, int T, int k, int d, cudaStream_t st) {
  if (T > 0) pdl_launch(prefill_combine, dim3(T), dim3(256), 0, st, ids, yret, x, T, k, d);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)f;
    cudaGetLastError();
  });
  return fn;
}

// f16 matrix [rows][cols] (row stride cols * 2 bytes), box {64, box_rows}, 128-byte swizzle
static int make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return VIREO_ERR_UNSUPPORTED;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? VIREO_OK : VIREO_ERR_UNSUPPORTED;
}

int prefill_supported(int d, int fe, int ne, int k, uint32_t rt, uint32_t gt, uint32_t ut, uint32_t dt) {
  return rt == T_F32 && gt == T_Q4_K && ut == T_Q4_K && dt == T_Q6_K && d % 256 == 0 && fe % 256 == 0 &&
         ne >= 1 && ne <= 128 && k >= 1 && k <= kPTopK && d <= 16384 && fe <= 16384;
}

void prefill_scratch_free(PrefillScratch* s) {
  for (void* p : {(void*)s->xa, (void*)s->ids, (void*)s->wts, (void*)s->counts, (void*)s->cursor, (void*)s->tiles,
                  (void*)s->n_mtiles, (void*)s->ysrc, (void*)s->wrow, (void*)s->xg, (void*)s->hg, (void*)s->yret,
                  (void*)s->r2, (void*)s->minmat, (void*)s->gu_pack, (void*)s->dn_pack})
    if (p) cudaFree(p);
  *s = PrefillScratch();
}

static int grow(void** p, size_t* cap, size_t bytes) {
  bytes = std::max<size_t>(bytes, 256);
  if (*cap >= bytes && *p) return VIREO_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return VIREO_ERR_NOMEM;
  }
  *cap = bytes;
  return VIREO_OK;
}

int prefill_kx(int d) { return d + ((d / 32 + 63) / 64) * 64; }
int prefill_tile_rows() { return kPM; }

static void set_attrs_once() {
  static std::once_flag attr_once;
  std::call_once(attr_once, [] {
    cudaFuncSetAttribute(prefill_gemm<P_ROUTER>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem<P_ROUTER>());
    cudaFuncSetAttribute(prefill_gemm<P_GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem<P_GATEUP>());
    cudaFuncSetAttribute(prefill_gemm<P_DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem<P_DOWN>());
  });
}

static PrefillParams base_params(const PrefillLayer& L, PrefillScratch* S, int T, int* d_err) {
  PrefillParams p;
  memset(&p, 0, sizeof(p));
  p.T = T;
  p.d = L.d;
  p.fe = L.fe;
  p.ne = L.ne;
  p.k = L.k;
  p.renorm = L.renorm;
  p.Kx = prefill_kx(L.d);
  p.exp_tab = L.exp_tab;
  p.rb_gu = (uint32_t)(L.d / 256 * 144);
  p.rb_d = (uint32_t)(L.fe / 256 * 210);
  p.ids = S->ids;
  p.wts = S->wts;
  p.counts = S->counts;
  p.n_mtiles = S->n_mtiles;
  p.tiles = S->tiles;
  p.hg = (__half*)S->hg;
  p.wrow = S->wrow;
  p.err = d_err;
  return p;
}

int prefill_prepare(const PrefillLayer& L, PrefillScratch* S, cudaStream_t st) {
  const int d = L.d, fe = L.fe, ne = L.ne;
  int rc;
  if (!S->r2) {
    if ((rc = grow((void**)&S->r2, &S->c_r2, (size_t)256 * d * 2))) return rc;
    prefill_router_split<<<256, 256, 0, st>>>(L.router, (__half*)S->r2, ne, d);
  }
  const int Km = prefill_kx(d) - d;
  if (!S->minmat_ok) {
    // per layer, once (again after the expert pointers change): the min block
    // and the repacked weight chunks the GEMMs stream, for the experts this
    // handle computes (L.own; all when null)
    const size_t n_gu = (size_t)ne * (fe / 128) * (d / kPK), n_dn = (size_t)ne * (d / kPN) * (fe / kPK);
    if ((rc = grow((void**)&S->minmat, &S->c_minmat, (size_t)ne * 2 * fe * Km * 2)) ||
        (rc = grow((void**)&S->gu_pack, &S->c_gu_pack, n_gu * kPRawGU)) ||
        (rc = grow((void**)&S->dn_pack, &S->c_dn_pack, n_dn * kPRawDN)))
      return rc;
    prefill_minmat<<<ne * 2 * fe, 64, 0, st>>>(L.exp_tab, L.own, d, fe, Km, (uint32_t)(d / 256 * 144), S->minmat);
    prefill_pack_gu<<<(unsigned)n_gu, kPN, 0, st>>>(L.exp_tab, L.own, d, fe, (uint32_t)(d / 256 * 144), S->gu_pack);
    prefill_pack_dn<<<(unsigned)n_dn, kPN, 0, st>>>(L.exp_tab, L.own, d, fe, (uint32_t)(fe / 256 * 210), S->dn_pack);
    S->minmat_ok = true;
  }
  return cuda_status(cudaGetLastError());
}

int prefill_route(const PrefillLayer& L, PrefillScratch* S, const void* hb, int T, const float* bias, int* d_err,
                  int num_sms, cudaStream_t st) {
  const int d = L.d, k = L.k, Kx = prefill_kx(d);
  const size_t pairs = (size_t)T * k;
  int rc;
  if ((rc = grow((void**)&S->xa, &S->c_xa, (size_t)T * Kx * 2)) || (rc = grow((void**)&S->ids, &S->c_ids, pairs * 4)) ||
      (rc = grow((void**)&S->wts, &S->c_wts, pairs * 4)) || (rc = grow((void**)&S->counts, &S->c_counts, 256 * 4)) ||
      (rc = grow((void**)&S->cursor, &S->c_cursor, 256 * 4)) || (rc = grow((void**)&S->n_mtiles, &S->c_n_mtiles, 16)))
    return rc;
  if ((rc = prefill_prepare(L, S, st))) return rc;
  CUtensorMap mA_r, mB_r;
  if ((rc = make_map(&mA_r, S->xa, T, Kx, kPM)) || (rc = make_map(&mB_r, S->r2, 256, d, kPN))) return rc;
  set_attrs_once();
  PrefillParams p = base_params(L, S, T, d_err);
  p.bias = bias;
  if ((rc = pdl_launch(prefill_prep, dim3(T), dim3(256), 0, st, (const __nv_bfloat16*)hb, (__half*)S->xa, T, d, Kx,
                       (int*)S->counts)))
    return rc;
  p.nk = d / kPK;
  // idle SMs repeat a row tile's GEMM so that its top-k is split 2 or 4 ways
  const int tiles = (T + kPM - 1) / kPM;
  p.n_ntiles = tiles * 4 <= num_sms ? 4 : tiles * 2 <= num_sms ? 2 : 1;
  return pdl_launch(prefill_gemm<P_ROUTER>, dim3(std::min(num_sms, tiles * p.n_ntiles)), dim3(kPThreads),
                    psmem<P_ROUTER>(), st, mA_r, mB_r, p);
  return cuda_status(cudaGetLastError());
}

size_t prefill_row_capacity(size_t pairs, int ne) { return ((pairs + (size_t)ne * (kPM - 1)) + kPM - 1) / kPM * kPM; }

int prefill_grow_rows(const PrefillLayer& L, PrefillScratch* S, size_t rows) {
  const int Kx = prefill_kx(L.d);
  rows = std::max<size_t>(rows, kPM);
  const size_t max_mtiles = rows / kPM + 1;
  int rc;
  if ((rc = grow((void**)&S->counts, &S->c_counts, 256 * 4)) || (rc = grow((void**)&S->cursor, &S->c_cursor, 256 * 4)) ||
      (rc = grow((void**)&S->n_mtiles, &S->c_n_mtiles, 16)) ||
      (rc = grow((void**)&S->tiles, &S->c_tiles, max_mtiles * sizeof(PTile))) ||
      (rc = grow((void**)&S->wrow, &S->c_wrow, rows * 4)) || (rc = grow((void**)&S->xg, &S->c_xg, rows * Kx * 2)) ||
      (rc = grow((void**)&S->hg, &S->c_hg, rows * L.fe * 2)))
    return rc;
  return VIREO_OK;
}

void prefill_scan_launch(const int* counts, int ne, PrefillScratch* S, cudaStream_t st) {
  pdl_launch(prefill_scan, dim3(1), dim3(256), 0, st, counts, ne, (int*)S->cursor, (PTile*)S->tiles, (int*)S->n_mtiles);
}

int prefill_experts(const PrefillLayer& L, PrefillScratch* S, size_t rows, int* d_err, int num_sms, cudaStream_t st,
                    const int* ysrc, __half* const* ypeer, int npeers) {
  if (npeers > kPMaxPeers) return VIREO_ERR_ARG;
  const int d = L.d, fe = L.fe, ne = L.ne, Kx = prefill_kx(d), Km = Kx - d;
  rows = std::max<size_t>(rows, kPM);
  CUtensorMap mA_gu, mA_d, mM;
  int rc;
  if ((rc = make_map(&mA_gu, S->xg, rows, Kx, 2 * kPM)) || (rc = make_map(&mA_d, S->hg, rows, fe, 2 * kPM)) ||
      (rc = make_map(&mM, S->minmat, (uint64_t)ne * 2 * fe, Km, 128)))
    return rc;
  set_attrs_once();
  PrefillParams p = base_params(L, S, 0, d_err);
  // gate/up + SwiGLU
  p.nk = Kx / kPK;
  p.n_ntiles = fe / 128;
  p.pack = S->gu_pack;
  if ((rc = pdl_launch(prefill_gemm<P_GATEUP>, dim3(num_sms), dim3(kPThreads), psmem<P_GATEUP>(), st, mA_gu, mM, p)))
    return rc;
  // down, scaled by the routing weight
  p.nk = fe / kPK;
  p.n_ntiles = d / kPN;
  p.pack = S->dn_pack;
  p.ysrc = ysrc;
  for (int i = 0; i < npeers; i++) p.ypeer[i] = ypeer[i];
  p.remote = npeers > 1;
  if ((rc = pdl_launch(prefill_gemm<P_DOWN>, dim3(num_sms), dim3(kPThreads), psmem<P_DOWN>(), st, mA_d, mA_d, p)))
    return rc;
  return cuda_status(cudaGetLastError());
}

int prefill_run(const PrefillLayer& L, PrefillScratch* S, const void* hb, float* x, int T, const float* bias,
                int32_t* ids_out, float* wts_out, int* d_err, int num_sms, cudaStream_t st) {
  const int d = L.d, ne = L.ne, k = L.k, Kx = prefill_kx(d);
  const size_t pairs = (size_t)T * k, rows = prefill_row_capacity(pairs, ne);
  int rc;
  if ((rc = prefill_route(L, S, hb, T, bias, d_err, num_sms, st))) return rc;
  if (pairs >= (1u << 24)) return VIREO_ERR_ARG;  // a return slot is 24 bits
  if ((rc = grow((void**)&S->ysrc, &S->c_ysrc, rows * 4)) || (rc = grow((void**)&S->yret, &S->c_yret, pairs * d * 2)) ||
      (rc = prefill_grow_rows(L, S, rows)))
    return rc;
  prefill_scan_launch(S->counts, ne, S, st);
  if ((rc = pdl_launch(prefill_place, dim3((unsigned)((pairs + 7) / 8)), dim3(256), 0, st, (const int32_t*)S->ids,
                       (const float*)S->wts, (const __half*)S->xa, T, k, Kx, (int*)S->cursor, (int*)S->ysrc,
                       (float*)S->wrow, (__half*)S->xg)))
    return rc;
  __half* const self[1] = {S->yret};
  if ((rc = prefill_experts(L, S, rows, d_err, num_sms, st, S->ysrc, self, 1))) return rc;
  prefill_combine_launch(S->ids, S->yret, x, T, k, d, st);
  if (ids_out && cudaMemcpyAsync(ids_out, S->ids, pairs * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return cuda_status(cudaGetLastError());
  if (wts_out && cudaMemcpyAsync(wts_out, S->wts, pairs * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return cuda_status(cudaGetLastError());
  return cuda_status(cudaGetLastError());
}

}  // namespace vireo
