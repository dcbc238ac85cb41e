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
//   scan     per-expert row ranges padded to 128, the table of 128-row tiles
//   place    every (token, slot) pair gets a row of its expert's range; the
//            token's xa row is copied there
//   gate/up  h = silu(X_e W_gate,e^T) * (X_e W_up,e^T) for every expert's rows
//            (tcgen05 GEMM, Q4_K weights dequantised to f16 in shared memory)
//   down     y = w_pair * (H_e W_down,e^T) (Q6_K weights, f16)
//   combine  x[t] += sum over rank t of y(t, slot), in rank order
//
// GEMM kernel (prefill_gemm<MODE>): persistent, one CTA per SM, 16 warps:
// warp 0 allocates TMEM (512 columns: two 128 x 256 fp32 accumulators) and
// issues the TMA loads of the activation tiles (128 rows x 64 K, 128-byte
// swizzle); warp 1 issues the tcgen05.mma (M 128, N 256, K 16) from one
// thread; warps 4-11 write the weight tiles (256 rows x 64 K) into shared
// memory, dequantising GGUF blocks straight into the swizzled f16 layout (the
// router's weight tile comes by TMA instead); warps 12-15 are the epilogue,
// reading their 32 TMEM lanes with tcgen05.ld.  A 4-stage ring of 48 KB
// stages (full / empty mbarriers) connects loads to MMAs; the two
// accumulators let the epilogue of one tile overlap the main loop of the
// next.  Every wait is bounded (kWaitLimitNs) and sets the status word.
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

#include "engine.cuh"
#include "moe_decode.cuh"
#include "umma.cuh"
#include "vireo_internal.h"

namespace vireo {

constexpr int kPM = 128;   // activation rows per tile
constexpr int kPN = 256;   // weight rows per tile
constexpr int kPK = 64;    // K per stage
constexpr int kPStages = 4;
constexpr int kPThreads = 512;
constexpr int kDqWarp0 = 4, kDqWarps = 8, kEpiWarp0 = 12;
constexpr int kPTopK = 8;  // prefill top-k limit (held in registers)
constexpr uint32_t kPStageA = kPM * kPK * 2, kPStageB = kPN * kPK * 2;
constexpr uint32_t kPSmem = 1024 + kPStages * (kPStageA + kPStageB);

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
  float* y;  // [rows][d]
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

// ---- Q4_K row -> 64 f16 of one K stage (gate/up B tiles) -------------------
// Values of chunk c of super-block sb, in the xa column order: positions
// 0..31 the low nibbles of qs[32c ..], 32..63 the high nibbles, each group of
// 4 ordered (0 2 1 3).  Value = round(d sc_j q); the -dmin m_j term is the
// min block.
VDEV void dq_q4k_stage(const uint8_t* rowp, int kt, int nkd, int d, uint8_t* tile, int r) {
  uint4 out[8];
  if (kt < nkd) {
    const uint8_t* sbp = rowp + (kt >> 2) * 144;
    const int c = kt & 3;
    const uint4 hd = __ldg(reinterpret_cast<const uint4*>(sbp));
    const uint4 qa = __ldg(reinterpret_cast<const uint4*>(sbp + 16 + 32 * c));
    const uint4 qb = __ldg(reinterpret_cast<const uint4*>(sbp + 32 + 32 * c));
    const float dd = h_lo(hd.x);
    uint32_t sc0, m0, sc1, m1;
    Q4K::scale_min(hd.y, hd.z, hd.w, 2 * c, sc0, m0);
    Q4K::scale_min(hd.y, hd.z, hd.w, 2 * c + 1, sc1, m1);
    const float a0f = dd * (float)sc0, a1f = dd * (float)sc1 * 0.0625f;  // high nibbles come as 16 q
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const bool fast = fabsf(a0f) < 32.f && fabsf(a1f) < 32.f;  // 1024 a exact in f16
    const __half2 A0 = __float2half2_rn(a0f), A1 = __float2half2_rn(a1f);
    const __half2 C0 = __hmul2(A0, __float2half2_rn(-1024.f)), C1 = __hmul2(A1, __float2half2_rn(-1024.f));
    const __half2 K1024 = __float2half2_rn(1024.f);
#pragma unroll
    for (int ch = 0; ch < 8; ch++) {
      const uint32_t msk = ch < 4 ? 0x000F000Fu : 0x00F000F0u;
      const __half2 A = ch < 4 ? A0 : A1, C = ch < 4 ? C0 : C1;
      const uint32_t w0 = w[2 * (ch & 3)], w1 = w[2 * (ch & 3) + 1];
      const uint32_t u[4] = {(w0 & msk) | 0x64006400u, ((w0 >> 8) & msk) | 0x64006400u, (w1 & msk) | 0x64006400u,
                             ((w1 >> 8) & msk) | 0x64006400u};
      uint32_t h[4];
#pragma unroll
      for (int i = 0; i < 4; i++)
        h[i] = fast ? h2u(__hfma2(u2h(u[i]), A, C)) : h2u(__hmul2(__hsub2(u2h(u[i]), K1024), A));
      out[ch] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  } else {
    // min block: column j (natural order) = -round(dmin m_j) of sub-block j
    const int jb = (kt - nkd) * 64;
#pragma unroll
    for (int ch = 0; ch < 8; ch++) {
      const int j0 = jb + 8 * ch, sb = j0 >> 3;
      uint32_t h[4] = {0u, 0u, 0u, 0u};
      if (sb < d / 256) {
        const uint4 hd = __ldg(reinterpret_cast<const uint4*>(rowp + sb * 144));
        const float dm = h_hi(hd.x);
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
          uint32_t sc, mn;
          Q4K::scale_min(hd.y, hd.z, hd.w, i, sc, mn);
          v[i] = -(dm * (float)mn);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) h[i] = h2u(__floats2half2_rn(v[2 * i], v[2 * i + 1]));
      }
      out[ch] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
#pragma unroll
  for (int ch = 0; ch < 8; ch++)
    *reinterpret_cast<uint4*>(tile + r * 128 + ((ch ^ (r & 7)) << 4)) = out[ch];
}

// n 32-bit words from a 2-byte-aligned global address (one extra word read)
template <int N>
VDEV void ldg_words_u16(const uint8_t* p, uint32_t (&w)[N]) {
  const uint32_t mis = (uint32_t)((uintptr_t)p & 3u);
  const uint32_t* q = reinterpret_cast<const uint32_t*>(p - mis);
  uint32_t raw[N + 1];
#pragma unroll
  for (int i = 0; i <= N; i++) raw[i] = __ldg(q + i);
#pragma unroll
  for (int i = 0; i < N; i++) w[i] = __funnelshift_r(raw[i], raw[i + 1], 8 * mis);
}

// ---- Q6_K row -> 64 f16 of one K stage (down B tiles) ----------------------
// Stage kt = quarter q of super-block sb: half h = q >> 1; positions 0..31
// stream s0 = 2 (q & 1), 32..63 stream s0 + 1 (values 64 q + l, 64 q + 32 + l
// of the super-block), groups of 4 ordered (0 2 1 3).  Value = round(d sc
// (z - 32)) with (1024 + z) - 1056 exact.
VDEV void dq_q6k_stage(const uint8_t* rowp, int kt, uint8_t* tile, int r) {
  const uint8_t* sbp = rowp + (kt >> 2) * 210;
  const int q = kt & 3, h = q >> 1, hi = q & 1, s0 = 2 * hi;
  uint32_t ql[16], qh[8];
  ldg_words_u16<16>(sbp + 64 * h, ql);
  ldg_words_u16<8>(sbp + 128 + 32 * h, qh);
  const float dd = __half2float(__ushort_as_half(
      (unsigned short)((uint32_t)__ldg(sbp + 208) | ((uint32_t)__ldg(sbp + 209) << 8))));
  const int8_t* sc = reinterpret_cast<const int8_t*>(sbp + 192 + 8 * h);
  const __half2 K1056 = __float2half2_rn(1056.f);
#pragma unroll
  for (int ch = 0; ch < 8; ch++) {
    const int s = s0 + (ch >> 2), l0 = 8 * (ch & 3);
    const __half2 A = __float2half2_rn(dd * (float)__ldg(sc + 2 * s + (l0 >> 4)));
    uint32_t hv[4];
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const uint32_t qlw = ql[(s & 1) * 8 + (l0 >> 2) + i], qhw = qh[(l0 >> 2) + i];
      const uint32_t z = ((qlw >> (4 * hi)) & 0x0F0F0F0Fu) | (((qhw >> (2 * s)) & 0x03030303u) << 4);
      const uint32_t u0 = (z & 0x00FF00FFu) | 0x64006400u, u1 = ((z >> 8) & 0x00FF00FFu) | 0x64006400u;
      hv[2 * i] = h2u(__hmul2(__hsub2(u2h(u0), K1056), A));
      hv[2 * i + 1] = h2u(__hmul2(__hsub2(u2h(u1), K1056), A));
    }
    *reinterpret_cast<uint4*>(tile + r * 128 + ((ch ^ (r & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  }
}

template <int MODE>
__global__ void __launch_bounds__(kPThreads, 1)
    prefill_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t praw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)praw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = sm;
  uint8_t* sB = sm + kPStages * kPStageA;
  __shared__ uint64_t full[kPStages], empty[kPStages], tfull[2], tempty[2], drain;
  __shared__ uint32_t tbase;
  __shared__ int n_items_s;
  __shared__ volatile int abort_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; s++) {
      mbar_init(&full[s], MODE == P_ROUTER ? 1u : 1u + kDqWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(&drain, 1);
    mbar_fence_init();
    abort_s = 0;
    n_items_s = MODE == P_ROUTER ? (p.T + kPM - 1) / kPM : (*p.n_mtiles) * p.n_ntiles;
  }
  if (warp == 0) tmem_alloc(&tbase, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tbase;
  const int n_items = n_items_s;
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
      // ---- TMA producer ------------------------------------------------------
      uint32_t g = 0;
      for (int item = blockIdx.x; item < n_items && !abort_s; item += gridDim.x) {
        const PTile t = tile_of(item / p.n_ntiles);
        for (int kt = 0; kt < p.nk; kt++, g++) {
          const int s = (int)(g % kPStages);
          if (g >= (uint32_t)kPStages && !pwait(&empty[s], ((g / kPStages) - 1) & 1, &abort_s, p.err)) break;
          mbar_arrive_expect_tx(&full[s], kPStageA + (MODE == P_ROUTER ? kPStageB : 0u));
          tma_load_2d(sA + s * kPStageA, &tmA, kt * kPK, t.row0, &full[s]);
          if constexpr (MODE == P_ROUTER) tma_load_2d(sB + s * kPStageB, &tmB, kt * kPK, 0, &full[s]);
        }
      }
      // the loads of the last stages land before the CTA may exit
      for (uint32_t j = g > (uint32_t)kPStages ? g - kPStages : 0; j < g; j++) {
        volatile int never = 0;
        mbar_wait(&full[j % kPStages], (j / kPStages) & 1, &never);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer --------------------------------------------------------
      constexpr uint32_t idesc = umma_idesc_f16(kPM, kPN);
      uint32_t g = 0;
      int it = 0;
      for (int item = blockIdx.x; item < n_items && !abort_s; item += gridDim.x, it++) {
        const int b = it & 1;
        if (it >= 2 && !pwait(&tempty[b], ((it >> 1) - 1) & 1, &abort_s, p.err)) break;
        tc_fence_after();
        const uint32_t dt = tmem + (uint32_t)(b * kPN);
        bool ok = true;
        for (int kt = 0; kt < p.nk; kt++, g++) {
          const int s = (int)(g % kPStages);
          if (!pwait(&full[s], (g / kPStages) & 1, &abort_s, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(sA + s * kPStageA), db = umma_desc_sw128(sB + s * kPStageB);
#pragma unroll
          for (int kk = 0; kk < kPK / 16; kk++)
            umma_f16_ss(dt, da + 2 * kk, db + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
      // every MMA issued here is complete before TMEM may be released
      umma_commit(&drain);
      volatile int never = 0;
      mbar_wait(&drain, 0, &never);
    }
  } else if (warp >= kDqWarp0 && warp < kDqWarp0 + kDqWarps) {
    if constexpr (MODE != P_ROUTER) {
      // ---- weight tiles: GGUF blocks -> swizzled f16 in shared memory --------
      const int r = threadIdx.x - 32 * kDqWarp0;  // tile row 0..255
      uint32_t g = 0;
      for (int item = blockIdx.x; item < n_items && !abort_s; item += gridDim.x) {
        const int mt = item / p.n_ntiles, nt = item - mt * p.n_ntiles;
        const PTile t = tile_of(mt);
        const uint8_t* rowp;
        if constexpr (MODE == P_GATEUP) {
          const int f = nt * 128 + (r & 127);
          rowp = p.exp_tab[3 * t.e + (r < 128 ? 0 : 1)] + (size_t)f * p.rb_gu;
        } else {
          rowp = p.exp_tab[3 * t.e + 2] + (size_t)(nt * kPN + r) * p.rb_d;
        }
        bool ok = true;
        for (int kt = 0; kt < p.nk; kt++, g++) {
          const int s = (int)(g % kPStages);
          int w_ok = 1;
          if (g >= (uint32_t)kPStages && lane == 0) w_ok = pwait(&empty[s], ((g / kPStages) - 1) & 1, &abort_s, p.err);
          w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
          if (!w_ok) {
            ok = false;
            break;
          }
          uint8_t* tile = sB + s * kPStageB;
          if constexpr (MODE == P_GATEUP) dq_q4k_stage(rowp, kt, p.d / kPK, p.d, tile, r);
          else dq_q6k_stage(rowp, kt, tile, r);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
        if (!ok) break;
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ---- epilogue ------------------------------------------------------------
    const int q = warp & 3;
    int it = 0;
    for (int item = blockIdx.x; item < n_items && !abort_s; item += gridDim.x, it++) {
      const int b = it & 1;
      int w_ok = 1;
      if (lane == 0) w_ok = pwait(&tfull[b], (it >> 1) & 1, &abort_s, p.err);
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      if (!w_ok) break;
      tc_fence_after();
      const int mt = item / p.n_ntiles, nt = item - mt * p.n_ntiles;
      const PTile t = tile_of(mt);
      const int rt = 32 * q + lane;  // row within the tile
      const bool valid = rt < t.nrows;
      const int row = t.row0 + rt;
      const uint32_t ta = tmem + (uint32_t)(b * kPN) + ((uint32_t)(32 * q) << 16);
      if constexpr (MODE == P_ROUTER) {
        // logits = hi + lo (+ bias); softmax; top-k; renorm  (gguf_run.c:187-192)
        const int ne = p.ne;
        float mx = -INFINITY;
        for (int c = 0; c < 128; c += 32) {
          uint32_t vh[32], vl[32];
          tmem_ld32(ta + c, vh);
          tmem_ld32(ta + 128 + c, vl);
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (c + j < ne) {
              const float l = __uint_as_float(vh[j]) + __uint_as_float(vl[j]) + (p.bias ? p.bias[c + j] : 0.f);
              mx = (j == 0 && c == 0) ? l : (l > mx ? l : mx);
            }
        }
        float sum = 0.f;
        for (int c = 0; c < 128; c += 32) {
          uint32_t vh[32], vl[32];
          tmem_ld32(ta + c, vh);
          tmem_ld32(ta + 128 + c, vl);
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (c + j < ne) {
              const float l = __uint_as_float(vh[j]) + __uint_as_float(vl[j]) + (p.bias ? p.bias[c + j] : 0.f);
              sum += expf(l - mx);
            }
        }
        float tv[kPTopK];
        int ti[kPTopK];
#pragma unroll
        for (int i = 0; i < kPTopK; i++) {
          tv[i] = -1.f;
          ti[i] = -1;
        }
        const int k = p.k;
        for (int c = 0; c < 128; c += 32) {
          uint32_t vh[32], vl[32];
          tmem_ld32(ta + c, vh);
          tmem_ld32(ta + 128 + c, vl);
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int e = c + j;
            if (e >= ne) continue;
            const float l = __uint_as_float(vh[j]) + __uint_as_float(vl[j]) + (p.bias ? p.bias[e] : 0.f);
            float pe = expf(l - mx) / sum;  // NaN never enters (strict '>')
            int pe_i = e;
#pragma unroll
            for (int i = 0; i < kPTopK; i++) {
              if (i < k && pe > tv[i]) {
                const float fv = tv[i];
                const int fi = ti[i];
                tv[i] = pe;
                ti[i] = pe_i;
                pe = fv;
                pe_i = fi;
              }
            }
          }
        }
        float ws = 0.f;
#pragma unroll
        for (int i = 0; i < kPTopK; i++)
          if (i < k) ws = ws + tv[i];
        if (valid) {
#pragma unroll
          for (int i = 0; i < kPTopK; i++) {
            if (i < k) {
              const float w = (p.renorm && ws > 0.f) ? tv[i] / ws : tv[i];
              p.ids[(size_t)row * k + i] = ti[i];
              p.wts[(size_t)row * k + i] = w;
              if (ti[i] >= 0) atomicAdd(&p.counts[ti[i]], 1);
            }
          }
        }
      } else if constexpr (MODE == P_GATEUP) {
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
              hv[i] = (g / (1.0f + expf(-g))) * u;
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
        // y = w * (H W_down^T), fp32
        const int n0 = nt * kPN;
        const float w = valid ? p.wrow[row] : 0.f;
#pragma unroll 1
        for (int c = 0; c < kPN; c += 32) {
          uint32_t v[32];
          tmem_ld32(ta + c, v);
          if (valid) {
            float4* dst = reinterpret_cast<float4*>(p.y + (size_t)row * p.d + n0 + c);
#pragma unroll
            for (int i = 0; i < 8; i++)
              dst[i] = make_float4(__uint_as_float(v[4 * i]) * w, __uint_as_float(v[4 * i + 1]) * w,
                                   __uint_as_float(v[4 * i + 2]) * w, __uint_as_float(v[4 * i + 3]) * w);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---- prep: xa[t] = [f16 of the token's values, columns (0 2 1 3) per group
// of 4 | f16 of the 32-value group sums | zero padding], Kx columns --------
__global__ void prefill_prep(const __nv_bfloat16* hb, __half* xa, int T, int d, int Kx) {
  const int t = blockIdx.x;
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

// ---- scan: padded row ranges, the tile table, placement cursors ------------
__global__ void prefill_scan(const int* counts, int ne, int* cursor, PTile* tiles, int* n_mtiles) {
  __shared__ int mts[256], offs[256];
  const int e = threadIdx.x;
  const int n = e < ne ? counts[e] : 0;
  mts[e] = (n + kPM - 1) / kPM;
  __syncthreads();
  if (e == 0) {
    int mt = 0, off = 0;
    for (int i = 0; i < ne; i++) {
      const int m = mts[i];
      mts[i] = mt;
      offs[i] = off;
      mt += m;
      off += m * kPM;
    }
    *n_mtiles = mt;
  }
  __syncthreads();
  if (e < ne) {
    cursor[e] = offs[e];
    for (int i = 0; i * kPM < n; i++) {
      PTile t;
      t.e = e;
      t.row0 = offs[e] + i * kPM;
      t.nrows = min(kPM, n - i * kPM);
      tiles[mts[e] + i] = t;
    }
  }
}

// ---- place: a row per (token, slot), the token's xa row copied there ------
__global__ void prefill_place(const int32_t* ids, const float* wts, const __half* xa, int T, int k, int Kx,
                              int* cursor, int* rowpos, float* wrow, __half* xg) {
  const int pair = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (pair >= T * k) return;
  int pos = -1;
  if (lane == 0) {
    const int e = ids[pair];
    if (e >= 0) {
      pos = atomicAdd(&cursor[e], 1);
      wrow[pos] = wts[pair];
    }
    rowpos[pair] = pos;
  }
  pos = __shfl_sync(0xffffffffu, pos, 0);
  if (pos < 0) return;
  const uint4* s = reinterpret_cast<const uint4*>(xa + (size_t)(pair / k) * Kx);
  uint4* dst = reinterpret_cast<uint4*>(xg + (size_t)pos * Kx);
  for (int i = lane; i < Kx / 8; i += 32) dst[i] = s[i];
}

// ---- combine: x[t] += sum over rank of y(t, slot) (gguf_run.c:209, 213) ----
__global__ void prefill_combine(const int* rowpos, const float* y, float* x, int T, int k, int d) {
  const int t = blockIdx.x;
  if (t >= T) return;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < k; i++) {
      const int r = rowpos[(size_t)t * k + i];
      if (r >= 0) acc = __fadd_rn(acc, y[(size_t)r * d + c]);
    }
    x[(size_t)t * d + c] = __fadd_rn(x[(size_t)t * d + c], acc);
  }
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
                  (void*)s->n_mtiles, (void*)s->rowpos, (void*)s->wrow, (void*)s->xg, (void*)s->hg, (void*)s->y,
                  (void*)s->r2})
    if (p) cudaFree(p);
  *s = PrefillScratch();
}

static int grow(void** p, size_t* cap, size_t bytes) {
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

int prefill_run(const PrefillLayer& L, PrefillScratch* S, const void* hb, float* x, int T, const float* bias,
                int32_t* ids_out, float* wts_out, int* d_err, int num_sms, cudaStream_t st) {
  const int d = L.d, fe = L.fe, ne = L.ne, k = L.k;
  const int Kx = d + ((d / 32 + 63) / 64) * 64;
  const size_t pairs = (size_t)T * k, rows = ((pairs + (size_t)ne * (kPM - 1)) + kPM - 1) / kPM * kPM;
  const size_t max_mtiles = rows / kPM + 1;
  int rc;
  if ((rc = grow((void**)&S->xa, &S->c_xa, (size_t)T * Kx * 2)) || (rc = grow((void**)&S->ids, &S->c_ids, pairs * 4)) ||
      (rc = grow((void**)&S->wts, &S->c_wts, pairs * 4)) || (rc = grow((void**)&S->counts, &S->c_counts, 256 * 4)) ||
      (rc = grow((void**)&S->cursor, &S->c_cursor, 256 * 4)) ||
      (rc = grow((void**)&S->tiles, &S->c_tiles, max_mtiles * sizeof(PTile))) ||
      (rc = grow((void**)&S->n_mtiles, &S->c_n_mtiles, 16)) || (rc = grow((void**)&S->rowpos, &S->c_rowpos, pairs * 4)) ||
      (rc = grow((void**)&S->wrow, &S->c_wrow, rows * 4)) || (rc = grow((void**)&S->xg, &S->c_xg, rows * Kx * 2)) ||
      (rc = grow((void**)&S->hg, &S->c_hg, rows * fe * 2)) || (rc = grow((void**)&S->y, &S->c_y, rows * d * 4)))
    return rc;
  if (!S->r2) {
    if ((rc = grow((void**)&S->r2, &S->c_r2, (size_t)256 * d * 2))) return rc;
    prefill_router_split<<<256, 256, 0, st>>>(L.router, (__half*)S->r2, ne, d);
  }
  CUtensorMap mA_r, mB_r, mA_gu, mA_d;
  if ((rc = make_map(&mA_r, S->xa, T, Kx, kPM)) || (rc = make_map(&mB_r, S->r2, 256, d, kPN)) ||
      (rc = make_map(&mA_gu, S->xg, rows, Kx, kPM)) || (rc = make_map(&mA_d, S->hg, rows, fe, kPM)))
    return rc;
  static std::once_flag attr_once;
  std::call_once(attr_once, [] {
    cudaFuncSetAttribute(prefill_gemm<P_ROUTER>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmem);
    cudaFuncSetAttribute(prefill_gemm<P_GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmem);
    cudaFuncSetAttribute(prefill_gemm<P_DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmem);
  });
  PrefillParams p;
  memset(&p, 0, sizeof(p));
  p.T = T;
  p.d = d;
  p.fe = fe;
  p.ne = ne;
  p.k = k;
  p.renorm = L.renorm;
  p.Kx = Kx;
  p.exp_tab = L.exp_tab;
  p.rb_gu = (uint32_t)(d / 256 * 144);
  p.rb_d = (uint32_t)(fe / 256 * 210);
  p.bias = bias;
  p.ids = S->ids;
  p.wts = S->wts;
  p.counts = S->counts;
  p.n_mtiles = S->n_mtiles;
  p.tiles = S->tiles;
  p.hg = (__half*)S->hg;
  p.wrow = S->wrow;
  p.y = S->y;
  p.err = d_err;

  if (cudaMemsetAsync(S->counts, 0, 256 * 4, st) != cudaSuccess) return cuda_status(cudaGetLastError());
  prefill_prep<<<T, 256, 0, st>>>((const __nv_bfloat16*)hb, (__half*)S->xa, T, d, Kx);
  // router
  p.nk = d / kPK;
  p.n_ntiles = 1;
  prefill_gemm<P_ROUTER><<<std::min(num_sms, (T + kPM - 1) / kPM), kPThreads, kPSmem, st>>>(mA_r, mB_r, p);
  prefill_scan<<<1, 256, 0, st>>>(S->counts, ne, S->cursor, S->tiles, S->n_mtiles);
  prefill_place<<<(unsigned)((pairs + 7) / 8), 256, 0, st>>>(S->ids, S->wts, (const __half*)S->xa, T, k, Kx,
                                                              S->cursor, S->rowpos, S->wrow, (__half*)S->xg);
  // gate/up + SwiGLU
  p.nk = Kx / kPK;
  p.n_ntiles = fe / 128;
  prefill_gemm<P_GATEUP><<<num_sms, kPThreads, kPSmem, st>>>(mA_gu, mA_gu, p);
  // down, scaled by the routing weight
  p.nk = fe / kPK;
  p.n_ntiles = d / kPN;
  prefill_gemm<P_DOWN><<<num_sms, kPThreads, kPSmem, st>>>(mA_d, mA_d, p);
  prefill_combine<<<T, 256, 0, st>>>(S->rowpos, S->y, x, T, k, d);
  if (ids_out && cudaMemcpyAsync(ids_out, S->ids, pairs * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return cuda_status(cudaGetLastError());
  if (wts_out && cudaMemcpyAsync(wts_out, S->wts, pairs * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return cuda_status(cudaGetLastError());
  return cuda_status(cudaGetLastError());
}

}  // namespace vireo
