// The decoder forward pass around the MoE block (include/gguf_decoder.h):
// one decode step of the reference's forward() (vireo src/gguf_run.c:216-252)
// on the device.  The projections and the LM head run on the quantised
// mat-vec engine of gguf_matmul_dev; the MoE block is gguf_moe_ffn; this file
// adds the small kernels in between: RMSNorm (fused with the residual add),
// the q/k post-processing (bias, QK norm, NEOX RoPE, KV append), exact
// attention over the KV cache (split over position chunks, merged with the
// online-softmax rule of the reference's KV store) and the greedy argmax.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <utility>
#include <vector>

#include "gguf_decoder.h"
#include "moe_view.h"
#include "vireo_internal.h"
#include "vireo_ptx.cuh"

namespace vireo {

constexpr int kDecThreads = 1024;
constexpr int kAttnChunk = 128;  // cached positions per attention CTA (one per thread)
constexpr int kCombThreads = 128;  // threads of the chunk-merging kernel
// positions a cache may hold: the merging kernel keeps a weight per chunk in
// (at most 48 KB of) shared memory
constexpr int kMaxCtx = (48 * 1024 / 4 - kCombThreads) * kAttnChunk;
// weight bytes per mat-vec CTA sent toward L2 before the CTA waits on the
// previous kernel
constexpr uint32_t kDecPrefetch = 128u << 10;

VDEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

VDEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// block-wide sum, every thread gets the total (blockDim.x a multiple of 32)
VDEV float block_sum(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; i++) t += red[i];
  return t;
}

// x (+)= y, then out = x * (1 / sqrt(mean(x^2) + eps)) * w  (rmsnorm,
// gguf_run.c:161-165; with y the residual add of gguf_run.c:237 first)
__global__ void __launch_bounds__(kDecThreads) dec_rmsnorm(float* x, const float* y, const float* w, float* out, int n,
                                                           float eps) {
  pdl_launch_dependents();  // the next kernel may take SMs now; it waits in its own prologue
  pdl_wait();  // inputs written by the previous kernel on the stream
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = x[i];
    if (y) {
      v = v + y[i];
      x[i] = v;
    }
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float r = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = x[i] * r * w[i];
}

// RMSNorm of one head (hs values in shared memory) by one warp:
// v * (1 / sqrt(ss / len + eps)) * w, with ss given (the head's own sum of
// squares for a per-head norm, the whole vector's for a full-width one)
VDEV void norm_head(float* v, int hs, const float* w, float ss, int len, float eps, int lane) {
  const float r = 1.0f / sqrtf(ss / (float)len + eps);
  for (int i = lane; i < hs; i += 32) v[i] = v[i] * r * w[i];
}

// sum of squares of (a[i] + b[i]) over n values (b may be null), block-wide
VDEV float block_sumsq(const float* a, const float* b, int n, float* red) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = b ? a[i] + b[i] : a[i];
    ss += v * v;
  }
  return block_sum(ss, red);
}

struct AttnParams {
  const float *q, *k, *v;     // this position's projections [nh hs], [nkv hs], [nkv hs]
  const float *bq, *bk, *bv;  // biases or null
  const float *qn, *kn;       // QK-norm weights or null
  int qn_len, kn_len;         // hs (per head) or the full width
  const float* freq;          // [hs / 2] RoPE frequencies, base^(-2j/hs)
  void *kc, *vc;              // this layer's caches, [nkv][max_ctx][hs]
  int nh, nkv, hs, pos, npos, max_ctx, nchunk;
  float scale, eps;
  float* part;  // [nh][nchunk][hs + 2]: acc, m, l
  int* err;     // status word (tensor-core path: a copy or a merge that timed out)
  unsigned int* cnt;  // tensor-core path: per kv head, [0] chunks written, [1] merges done (zero between launches)
  float* out;         // tensor-core path: the merged attention output [nh][hs]
};

VDEV float kv_load(const float* p, size_t i) { return p[i]; }
VDEV float kv_load(const __half* p, size_t i) { return __half2float(p[i]); }
VDEV void kv_store(float* p, size_t i, float v) { p[i] = v; }
VDEV void kv_store(__half* p, size_t i, float v) { p[i] = __float2half_rn(v); }

// 8 consecutive cache values starting at element i (i a multiple of 8)
VDEV void kv_load8(const float* p, size_t i, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p + i), b = *reinterpret_cast<const float4*>(p + i + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
VDEV void kv_load8(const __half* p, size_t i, float (&o)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p + i);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float2 f = __half22float2(h[j]);
    o[2 * j] = f.x;
    o[2 * j + 1] = f.y;
  }
}

// NEOX rotation of `nv` heads of HS values in place (rope_neox,
// gguf_run.c:168-173): pairs (j, j + HS/2) turned by pos * freq[j]
template <int HS>
VDEV void rope_heads(float* v, int nv, int pos, const float* freq, int tid = -1, int nthr = 0) {
  constexpr int half = HS / 2;
  if (tid < 0) {
    tid = threadIdx.x;
    nthr = blockDim.x;
  }
  for (int idx = tid; idx < nv * half; idx += nthr) {
    const int h = idx / half, j = idx - h * half;
    float* w = v + h * HS;
    const float a = (float)pos * freq[j];
    const float c = cosf(a), s = sinf(a);
    const float x0 = w[j], x1 = w[j + half];
    w[j] = x0 * c - x1 * s;
    w[j + half] = x0 * s + x1 * c;
  }
}

// Attention of one token, one (chunk of kAttnChunk positions, kv head) per
// CTA, with all QG q heads that share the kv head (GQA).
//
// Prologue (the token's q/k post-processing, done by each CTA for its own
// heads): bias (gguf_run.c:223-225), QK RMSNorm per head or over the full
// width (:226-229, :177-179), NEOX RoPE (:230-231); the CTA whose chunk
// holds position pos also appends this position's k and v to the cache
// (:232-233) and reads it back with the rest of its chunk.  The cached rows of
// earlier positions were written by earlier steps, so they are prefetched to
// L2 before the kernel waits on the projection kernel.
//
// Scores: thread (position t, head group) reads the position's key row once
// (HS/8 16-byte loads in flight) and scores it against the group's q heads
// (two groups of 128 threads when QG >= 2, so that each thread's chain of
// FMAs is half as long and an SM holds twice the warps).  The chunk's softmax
// state per q head is formed (max, exp, sum).  Values: thread (dg, pg)
// accumulates dimensions 8 dg .. 8 dg + 7 over positions pg, pg + PG, ...
// with 16-byte loads, and the position groups are summed.  The state
// (acc, m, l) of each (q head, chunk) goes to part and dec_attn_combine
// merges the chunks: the reference's softmax attention (kvstore.h:77-101)
// evaluated chunk-parallel instead of one position at a time.
template <class KT, int QG, int HS, int SPLIT>
__global__ void __launch_bounds__(kAttnChunk* SPLIT) dec_attn_partial(const __grid_constant__ AttnParams p) {
  // SPLIT groups of kAttnChunk threads; in the score phase group hg scores
  // every position of the chunk against q heads hg QH .. hg QH + QH - 1
  constexpr int NT = kAttnChunk * SPLIT, QH = QG / SPLIT, NWG = kAttnChunk / 32, NW = NT / 32;
  constexpr int DG = HS / 8, PG = NT / DG;
  static_assert(QG % SPLIT == 0, "heads split evenly over the groups");
  __shared__ __align__(16) float sq[QG][HS];
  __shared__ __align__(16) float skv[2][HS];  // this position's k and v
  __shared__ float sp[QG][kAttnChunk];
  __shared__ float redm[QG][NWG], reds[QG][NWG];
  __shared__ float bred[32];
  __shared__ float racc[NW][QG * HS];
  const int c = blockIdx.x, kh = blockIdx.y, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int h0 = kh * QG;
  KT* kb = reinterpret_cast<KT*>(p.kc) + (size_t)kh * p.max_ctx * HS;
  KT* vb = reinterpret_cast<KT*>(p.vc) + (size_t)kh * p.max_ctx * HS;
  const int n = min(kAttnChunk, p.npos - c * kAttnChunk);
  const int cur = p.pos - c * kAttnChunk;  // this position's row in the chunk
  const bool has_cur = cur >= 0 && cur < n;
  if (t == 0) {
    const int nold = has_cur ? cur : n;
    if (nold > 0) {
      const size_t at = (size_t)c * kAttnChunk * HS;
      prefetch_l2(kb + at, (uint32_t)(nold * HS * sizeof(KT)));
      prefetch_l2(vb + at, (uint32_t)(nold * HS * sizeof(KT)));
    }
  }
  pdl_launch_dependents();  // the next kernel may take SMs now; it waits in its own prologue
  pdl_wait();               // q, k, v written by the projection kernel

  // ---- q heads h0 .. h0 + QG - 1 (and this position's k, v): bias, norm, rotation
  for (int i = t; i < QG * HS; i += NT) {
    const size_t gi = (size_t)h0 * HS + i;
    sq[i / HS][i % HS] = p.bq ? p.q[gi] + p.bq[gi] : p.q[gi];
  }
  if (has_cur)
    for (int i = t; i < HS; i += NT) {
      const size_t gi = (size_t)kh * HS + i;
      skv[0][i] = p.bk ? p.k[gi] + p.bk[gi] : p.k[gi];
      skv[1][i] = p.bv ? p.v[gi] + p.bv[gi] : p.v[gi];
    }
  // full-width norms need the whole vector's sum of squares
  float qss = 0.f, kss = 0.f;
  if (p.qn && p.qn_len != HS) qss = block_sumsq(p.q, p.bq, p.qn_len, bred);
  if (has_cur && p.kn && p.kn_len != HS) {
    __syncthreads();
    kss = block_sumsq(p.k, p.bk, p.kn_len, bred);
  }
  __syncthreads();
  if (p.qn) {
    for (int g = warp; g < QG; g += NW) {
      float ss = qss;
      if (p.qn_len == HS) {
        ss = 0.f;
        for (int i = lane; i < HS; i += 32) ss += sq[g][i] * sq[g][i];
        ss = warp_sum(ss);
      }
      norm_head(sq[g], HS, p.qn_len == HS ? p.qn : p.qn + (size_t)(h0 + g) * HS, ss, p.qn_len, p.eps, lane);
    }
  }
  if (has_cur && p.kn && warp == NW - 1) {
    float ss = kss;
    if (p.kn_len == HS) {
      ss = 0.f;
      for (int i = lane; i < HS; i += 32) ss += skv[0][i] * skv[0][i];
      ss = warp_sum(ss);
    }
    norm_head(skv[0], HS, p.kn_len == HS ? p.kn : p.kn + (size_t)kh * HS, ss, p.kn_len, p.eps, lane);
  }
  __syncthreads();
  rope_heads<HS>(&sq[0][0], QG, p.pos, p.freq);
  if (has_cur) rope_heads<HS>(skv[0], 1, p.pos, p.freq);
  __syncthreads();
  if (has_cur) {
    // append to the cache; after the barrier the chunk reads the row back
    // like every other (coherent loads: the same pointers are stored to)
    for (int i = t; i < HS; i += NT) {
      const size_t at = (size_t)p.pos * HS + i;
      kv_store(kb, at, skv[0][i]);
      kv_store(vb, at, skv[1][i]);
    }
    __syncthreads();
  }

  // ---- scores: thread (position pp, head group hg)
  const int pp = t % kAttnChunk, hg = t / kAttnChunk, wg = pp >> 5;
  const bool live = pp < n;
  float s[QH];
#pragma unroll
  for (int g = 0; g < QH; g++) s[g] = 0.f;
  if (live) {
    const size_t row = ((size_t)c * kAttnChunk + pp) * HS;
#pragma unroll
    for (int i = 0; i < HS; i += 8) {
      float e[8];
      kv_load8(kb, row + i, e);
#pragma unroll
      for (int g = 0; g < QH; g++)
#pragma unroll
        for (int j = 0; j < 8; j++) s[g] += sq[hg * QH + g][i + j] * e[j];
    }
  }
  // chunk max and sum per q head (over the NWG warps of the head's group)
#pragma unroll
  for (int g = 0; g < QH; g++) {
    const float v = live ? s[g] * p.scale : -INFINITY;
    s[g] = v;
    const float m = warp_max(v);
    if (lane == 0) redm[hg * QH + g][wg] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < QH; g++) {
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWG; w++) m = fmaxf(m, redm[hg * QH + g][w]);
    const float e = live ? expf(s[g] - m) : 0.f;
    sp[hg * QH + g][pp] = e;
    const float v = warp_sum(e);
    if (lane == 0) reds[hg * QH + g][wg] = v;
  }
  __syncthreads();
  // values: thread (dg, pg), 8 dimensions x the chunk's positions pg + PG u,
  // every q head
  const int dg = t % DG, pg = t / DG;
  float acc[QG][8];
#pragma unroll
  for (int g = 0; g < QG; g++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[g][j] = 0.f;
  const size_t vbase = (size_t)c * kAttnChunk * HS + 8 * dg;
#pragma unroll 4
  for (int u = pg; u < n; u += PG) {
    float v[8];
    kv_load8(vb, vbase + (size_t)u * HS, v);
#pragma unroll
    for (int g = 0; g < QG; g++) {
      const float w = sp[g][u];
#pragma unroll
      for (int j = 0; j < 8; j++) acc[g][j] += w * v[j];
    }
  }
  // sum the position groups: lanes with the same dg within a warp, then warps
#pragma unroll
  for (int o = DG; o < 32; o <<= 1)
#pragma unroll
    for (int g = 0; g < QG; g++)
#pragma unroll
      for (int j = 0; j < 8; j++) acc[g][j] += __shfl_xor_sync(0xffffffffu, acc[g][j], o);
  if (lane < DG)
#pragma unroll
    for (int g = 0; g < QG; g++)
#pragma unroll
      for (int j = 0; j < 8; j++) racc[warp][g * HS + 8 * dg + j] = acc[g][j];
  __syncthreads();
  for (int i = t; i < QG * HS; i += NT) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NW; w++) a += racc[w][i];
    const int g = i / HS, e = i - g * HS;
    p.part[((size_t)(h0 + g) * p.nchunk + c) * (HS + 2) + e] = a;
  }
  if (t < QG) {
    float M = -INFINITY, L = 0.f;
#pragma unroll
    for (int w = 0; w < NWG; w++) {
      M = fmaxf(M, redm[t][w]);
      L += reds[t][w];
    }
    float* out = p.part + ((size_t)(h0 + t) * p.nchunk + c) * (HS + 2);
    out[HS] = M;
    out[HS + 1] = L;
  }
}

// ---------------------------------------------------------------------------
// Tensor-core attention over the f16 KV cache: one CTA per (chunk of
// positions, kv head), four consumer warps and one producer warp.
//
// The f16 cache rows are stored swizzled: the 16-byte chunk c of position
// p's row sits at chunk c ^ (p & 7) (kv_swz), so that 8 consecutive
// positions read at the same logical chunk fall on 8 distinct bank groups.
// The producer streams the chunk's cached K and V rows in tiles of kAttnTile
// positions into a ring of shared-memory stages, one 1-D bulk copy for a
// tile's K rows and one for its V rows (the rows are contiguous in the
// cache).  Consumer warp w takes rows 16 w .. 16 w + 15 of every tile:
//   scores  S = Q K^T with mma.m16n8k16 (f16 in, fp32 accumulate): the QG q
//           heads of the kv group are the M rows (rows QG..15 zero), 8
//           positions are the N columns, K is the head dimension; the K rows
//           load as B fragments with ldmatrix.  Q carries the 1/sqrt(HS)
//           scale.
//   softmax per head over the warp's positions, online across tiles (the
//           reference's running max / sum rule, kvstore.h:77-101), in fp32;
//   values  O += P V with the score accumulators of two position tiles
//           reused as the A fragment (P rounded to f16) and the V rows loaded
//           transposed (ldmatrix.trans) as B fragments.
// The four warps' states are merged in shared memory and the CTA's state per
// q head (acc, m, l) goes to part; dec_attn_combine merges the chunks.
// The q/k post-processing and the KV append are those of dec_attn_partial.
// ---------------------------------------------------------------------------
constexpr int kAttnTile = 64;   // positions per stage
constexpr int kAttnWarps = 4;   // consumer warps, 16 positions of a tile each
constexpr int kAttnStages = 3;
constexpr int kAttnMmaThreads = 32 * (kAttnWarps + 1);

template <int HS>
struct AttnMmaLayout {
  static constexpr int kRow = HS * 2;               // f16 row bytes
  static constexpr int kStage = 2 * kAttnTile * kRow;  // K rows then V rows
  static constexpr int kOffQ = 64;                  // after the barriers
};

// element index inside a swizzled f16 cache row of position pos: dimension
// e's 16-byte chunk is stored at chunk (e / 8) ^ (pos & 7)
VDEV int kv_swz(int e, int pos) { return ((((e >> 3) ^ (pos & 7))) << 3) | (e & 7); }

template <int QG, int HS>
constexpr size_t attn_mma_smem() {
  using Ly = AttnMmaLayout<HS>;
  size_t off = Ly::kOffQ + sizeof(float) * (QG * HS + 2 * HS + 32 + 8);
  off += sizeof(float) * kAttnWarps * QG * (HS + 2);  // warp states for the merge
  off += sizeof(float) * (2 * QG * HS + 4 * HS + 4 * QG);  // RoPE table, norm weights, biases, merge weights
  off = (off + 127) / 128 * 128;
  return off + (size_t)kAttnStages * Ly::kStage;
}

template <int QG, int HS>
__global__ void __launch_bounds__(kAttnMmaThreads) dec_attn_mma(const __grid_constant__ AttnParams p, int C) {
  using Ly = AttnMmaLayout<HS>;
  constexpr int NC = 32 * kAttnWarps;  // consumer threads
  constexpr int KS = HS / 16;          // k16 steps of the scores
  constexpr int NT = HS / 8;           // n8 tiles of the values
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm);
  uint64_t* empty = full + kAttnStages;
  float* sq = reinterpret_cast<float*>(sm + Ly::kOffQ);  // [QG][HS] q heads
  float* skv = sq + QG * HS;                             // [2][HS] this position's k, v
  float* bred = skv + 2 * HS;                            // [32]
  int* flags = reinterpret_cast<int*>(bred + 32);        // [8]: abort, last
  float* wst = bred + 40;                                // [warps][QG][HS + 2] warp states
  float* rcs = wst + kAttnWarps * QG * (HS + 2);         // [HS]: cos, then sin, of pos * freq[j]
  float* wqs = rcs + HS;                                 // [QG][HS] q norm weights (per head: [HS])
  float* wks = wqs + QG * HS;                            // [HS] k norm weights
  float* bqs = wks + HS;                                 // [QG][HS] q bias (0 without one)
  float* bks = bqs + QG * HS;                            // [HS] k bias
  float* bvs = bks + HS;                                 // [HS] v bias
  float* mw = bvs + HS;                                  // [kAttnWarps][QG] merge weights
  uint8_t* ring = sm + ((Ly::kOffQ + sizeof(float) * (QG * HS + 2 * HS + 40 + kAttnWarps * QG * (HS + 2) +
                                                      2 * QG * HS + 4 * HS + 4 * QG) + 127) /
                        128 * 128);
  const int c = blockIdx.x, kh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h0 = kh * QG;
  __half* kb = reinterpret_cast<__half*>(p.kc) + (size_t)kh * p.max_ctx * HS;
  __half* vb = reinterpret_cast<__half*>(p.vc) + (size_t)kh * p.max_ctx * HS;
  const int p0 = c * C, n = min(C, p.npos - p0);
  const int cur = p.pos - p0;  // this position's row in the chunk (the chunk's last, if it holds it)
  const bool has_cur = cur >= 0 && cur < n;
  const int nold = has_cur ? cur : n;  // cached rows to stream
  const int ntile = (n + kAttnTile - 1) / kAttnTile;
  if (tid == 0) {
    for (int s = 0; s < kAttnStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kAttnWarps);
    }
    flags[0] = 0;
    mbar_fence_init();
    if (nold > 0) {
      prefetch_l2(kb + (size_t)p0 * HS, (uint32_t)(nold * HS * 2));
      prefetch_l2(vb + (size_t)p0 * HS, (uint32_t)(nold * HS * 2));
    }
  }
  // weights and this position's RoPE table (independent of the previous
  // kernel), staged while the projection kernel finishes
  if (tid < NC) {
    for (int j = tid; j < HS / 2; j += NC) {
      const float a = (float)p.pos * p.freq[j];
      rcs[j] = cosf(a);
      rcs[HS / 2 + j] = sinf(a);
    }
    const bool qfull = p.qn && p.qn_len != HS, kfull = p.kn && p.kn_len != HS;
    for (int i = tid; i < QG * HS; i += NC) {
      const size_t gi = (size_t)h0 * HS + i;
      bqs[i] = p.bq ? p.bq[gi] : 0.f;
      if (p.qn) wqs[i] = qfull ? p.qn[gi] : p.qn[i % HS];
    }
    for (int i = tid; i < HS; i += NC) {
      const size_t gi = (size_t)kh * HS + i;
      bks[i] = p.bk ? p.bk[gi] : 0.f;
      bvs[i] = p.bv ? p.bv[gi] : 0.f;
      if (p.kn) wks[i] = kfull ? p.kn[gi] : p.kn[i];
    }
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();  // q, k, v written by the projection kernel; earlier rows by earlier steps

  if (warp == kAttnWarps) {
    // ---- producer: the chunk's cached rows, tile by tile ----------------------
    int i = 0;
    for (; i < ntile; i++) {
      const int slot = i % kAttnStages;
      if (i >= kAttnStages) {
        int ok = 1;
        if (lane == 0) ok = mbar_wait(&empty[slot], ((uint32_t)(i / kAttnStages) & 1u) ^ 1u, flags) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      const int r0 = i * kAttnTile, rows = max(0, min(kAttnTile, nold - r0));
      uint8_t* st = ring + (size_t)slot * Ly::kStage;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(2 * rows * HS * 2));
        if (rows > 0) {
          const size_t g = (size_t)(p0 + r0) * HS;
          bulk_g2s(st, kb + g, (uint32_t)(rows * HS * 2), &full[slot]);
          bulk_g2s(st + (size_t)kAttnTile * Ly::kRow, vb + g, (uint32_t)(rows * HS * 2), &full[slot]);
        }
      }
    }
    // no copy may still be landing when the CTA exits
    if (lane == 0) {
      const int never = 0;
      for (int j = i > kAttnStages ? i - kAttnStages : 0; j < i; j++)
        mbar_wait(&full[j % kAttnStages], (uint32_t)(j / kAttnStages) & 1u, &never);
    }
    __syncwarp();
    return;
  }

  // ---- consumers: q heads h0 .. h0 + QG - 1 (and this position's k, v) -------
  for (int i = tid; i < QG * HS; i += NC) sq[i] = p.q[(size_t)h0 * HS + i] + bqs[i];
  if (has_cur)
    for (int i = tid; i < HS; i += NC) {
      const size_t gi = (size_t)kh * HS + i;
      skv[i] = p.k[gi] + bks[i];
      skv[HS + i] = p.v[gi] + bvs[i];
    }
  // full-width norms need the whole vector's sum of squares
  float qss = 0.f, kss = 0.f;
  if (p.qn && p.qn_len != HS) {
    float v = 0.f;
    for (int i = tid; i < p.qn_len; i += NC) {
      const float a = p.bq ? p.q[i] + p.bq[i] : p.q[i];
      v += a * a;
    }
    v = warp_sum(v);
    if (lane == 0) bred[warp] = v;
    asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
    for (int w = 0; w < kAttnWarps; w++) qss += bred[w];
    asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  }
  if (has_cur && p.kn && p.kn_len != HS) {
    float v = 0.f;
    for (int i = tid; i < p.kn_len; i += NC) {
      const float a = p.bk ? p.k[i] + p.bk[i] : p.k[i];
      v += a * a;
    }
    v = warp_sum(v);
    if (lane == 0) bred[warp] = v;
    asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
    for (int w = 0; w < kAttnWarps; w++) kss += bred[w];
    asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  }
  asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  if (p.qn)
    for (int g = warp; g < QG; g += kAttnWarps) {
      float ss = qss;
      if (p.qn_len == HS) {
        ss = 0.f;
        for (int i = lane; i < HS; i += 32) ss += sq[g * HS + i] * sq[g * HS + i];
        ss = warp_sum(ss);
      }
      norm_head(sq + g * HS, HS, wqs + g * HS, ss, p.qn_len, p.eps, lane);
    }
  if (has_cur && p.kn && warp == kAttnWarps - 1) {
    float ss = kss;
    if (p.kn_len == HS) {
      ss = 0.f;
      for (int i = lane; i < HS; i += 32) ss += skv[i] * skv[i];
      ss = warp_sum(ss);
    }
    norm_head(skv, HS, wks, ss, p.kn_len, p.eps, lane);
  }
  asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  // NEOX RoPE from the staged table
  for (int idx = tid; idx < (QG + (has_cur ? 1 : 0)) * (HS / 2); idx += NC) {
    const int hh = idx / (HS / 2), j = idx - hh * (HS / 2);
    float* w = hh < QG ? sq + hh * HS : skv;
    const float c = rcs[j], sn = rcs[HS / 2 + j];
    const float x0 = w[j], x1 = w[j + HS / 2];
    w[j] = x0 * c - x1 * sn;
    w[j + HS / 2] = x0 * sn + x1 * c;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  if (has_cur)  // the cache row later steps read (swizzled)
    for (int i = tid; i < HS; i += NC) {
      kb[(size_t)p.pos * HS + kv_swz(i, p.pos)] = __float2half_rn(skv[i]);
      vb[(size_t)p.pos * HS + kv_swz(i, p.pos)] = __float2half_rn(skv[HS + i]);
    }

  // Q as A fragments, scaled: row g (a q head when g < QG), rows g + 8 zero
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t qa[KS][2];
#pragma unroll
  for (int s = 0; s < KS; s++) {
    if (g < QG) {
      const float* q = sq + g * HS + 16 * s + 2 * t4;
      qa[s][0] = pack_h2(q[0] * p.scale, q[1] * p.scale);
      qa[s][1] = pack_h2(q[8] * p.scale, q[9] * p.scale);
    } else {
      qa[s][0] = qa[s][1] = 0u;
    }
  }
  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

#pragma unroll 1
  for (int i = 0; i < ntile; i++) {
    const int slot = i % kAttnStages;
    int ok = 1;
    if (lane == 0) ok = mbar_wait(&full[slot], (uint32_t)(i / kAttnStages) & 1u, flags) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    if (!ok && lane == 0 && !flags[0]) {
      flags[0] = 1;
      set_error(p.err, VIREO_ERR_TIMEOUT);
    }
    uint8_t* st = ring + (size_t)slot * Ly::kStage;
    const int rows = min(kAttnTile, n - i * kAttnTile);  // positions of this tile
    const int wr = 16 * warp;                             // this warp's first row
    if (ok && wr < rows) {
      // rows the copies did not fill: this position's k, v (from the q/k
      // step, f16) and, past the chunk's end, zeros (P = 0 cannot cancel a
      // NaN left in shared memory)
      const int last = (n - 1) - i * kAttnTile;  // the chunk's last row in this tile, if it is here
      for (int r = wr; r < wr + 16; r++) {
        const bool is_cur = has_cur && r == cur - i * kAttnTile;
        if (r < rows && !is_cur) continue;
        __half* kr = reinterpret_cast<__half*>(st + (size_t)r * Ly::kRow);
        __half* vr = reinterpret_cast<__half*>(st + (size_t)(kAttnTile + r) * Ly::kRow);
        for (int e = lane; e < HS; e += 32) {
          const int se = kv_swz(e, r);  // the tile's rows start at a multiple of 8 positions
          kr[se] = is_cur ? __float2half_rn(skv[e]) : __float2half_rn(0.f);
          vr[se] = is_cur ? __float2half_rn(skv[HS + e]) : __float2half_rn(0.f);
        }
      }
      (void)last;
      // generic writes into a stage that bulk copies also write
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      // scores of positions wr .. wr + 15: two n8 tiles
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < KS; s += 2) {
        uint32_t b[2][4];
#pragma unroll
        for (int j = 0; j < 2; j++) {
          const int r = wr + 8 * j + (lane & 7), ch = 2 * s + (lane >> 3);
          const uint8_t* row = st + (size_t)r * Ly::kRow + 16 * (ch ^ (r & 7));
          ldsm_x4(row, b[j][0], b[j][1], b[j][2], b[j][3]);
        }
        uint32_t a0[4] = {qa[s][0], 0u, qa[s][1], 0u}, a1[4] = {qa[s + 1][0], 0u, qa[s + 1][1], 0u};
        mma_16816(s0, a0, b[0][0], b[0][1]);
        mma_16816(s0, a1, b[0][2], b[0][3]);
        mma_16816(s1, a0, b[1][0], b[1][1]);
        mma_16816(s1, a1, b[1][2], b[1][3]);
      }
      // positions of this lane's scores: wr + 2 t4 (+1) and wr + 8 + 2 t4 (+1)
      const int q0 = wr + 2 * t4;
      float v0 = q0 < rows ? s0[0] : -INFINITY, v1 = q0 + 1 < rows ? s0[1] : -INFINITY;
      float v2 = q0 + 8 < rows ? s1[0] : -INFINITY, v3 = q0 + 9 < rows ? s1[1] : -INFINITY;
      float mt = fmaxf(fmaxf(v0, v1), fmaxf(v2, v3));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      const float m_new = fmaxf(m_run, mt);  // finite: the warp's first row is a position
      const float alpha = expf(m_run - m_new);
      const float e0 = expf(v0 - m_new), e1 = expf(v1 - m_new), e2 = expf(v2 - m_new), e3 = expf(v3 - m_new);
      l_run = l_run * alpha + ((e0 + e1) + (e2 + e3));
      m_run = m_new;
#pragma unroll
      for (int j = 0; j < NT; j++) {
        o[j][0] *= alpha;
        o[j][1] *= alpha;
      }
      const uint32_t pa[4] = {pack_h2(e0, e1), 0u, pack_h2(e2, e3), 0u};
      // values: O[g][8 j + 2 t4 ..] += P V
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = wr + (lane & 7) + 8 * ((lane >> 3) & 1), ch = j + (lane >> 4);
        const uint8_t* row = st + (size_t)(kAttnTile + r) * Ly::kRow + 16 * (ch ^ (r & 7));
        ldsm_x4_trans(row, b0, b1, b2, b3);
        mma_16816(o[j], pa, b0, b1);
        mma_16816(o[j + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  // ---- the four warps' states (row g = q head g) merged in shared memory ------
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  float* ws = wst + (size_t)warp * QG * (HS + 2);
  if (g < QG) {
#pragma unroll
    for (int j = 0; j < NT; j++) {
      ws[g * (HS + 2) + 8 * j + 2 * t4] = o[j][0];
      ws[g * (HS + 2) + 8 * j + 2 * t4 + 1] = o[j][1];
    }
    if (t4 == 0) {
      ws[g * (HS + 2) + HS] = m_run;
      ws[g * (HS + 2) + HS + 1] = l_run;
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  // per (warp, head) weights exp(m_w - M) once, then the weighted sums
  if (tid < kAttnWarps * QG) {
    const int w = tid / QG, h = tid - w * QG;
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < kAttnWarps; u++) M = fmaxf(M, wst[(u * QG + h) * (HS + 2) + HS]);
    const float m1 = wst[(w * QG + h) * (HS + 2) + HS];
    mw[tid] = m1 > -INFINITY ? expf(m1 - M) : 0.f;
    if (w == 0) bred[h] = M;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  float* cp = p.part + (size_t)h0 * p.nchunk * (HS + 2);
  for (int idx = tid; idx < QG * (HS + 2); idx += NC) {
    const int h = idx / (HS + 2), e = idx - h * (HS + 2);
    float a = 0.f;
    if (e == HS) {
      a = bred[h];
    } else {
#pragma unroll
      for (int w = 0; w < kAttnWarps; w++) a += wst[(w * QG + h) * (HS + 2) + e] * mw[w * QG + h];
    }
    cp[((size_t)h * p.nchunk + c) * (HS + 2) + e] = a;
  }

  // ---- the chunk merge (kv_softmax_finish, kvstore.h:99-101) -----------------
  // Once every chunk of this kv head has written its state, CTAs c <
  // min(QG, nchunk) of the kv head merge its q heads h0 + c, h0 + c + nchunk,
  // ...: thread e on dimension e, every chunk's value in flight at once, the
  // weights exp(m_c - M) and L = sum l_c exp(m_c - M) in chunk order.  The
  // last merging CTA puts the two counters back to zero.
  const int nc = p.nchunk, nmerge = min(QG, nc);
  __threadfence();
  asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  if (tid == 0) red_add_release_gpu(&p.cnt[2 * kh], 1u);
  if (c >= nmerge) return;
  if (tid == 0) flags[1] = wait_geq(&p.cnt[2 * kh], (unsigned)nc, p.err) ? 1 : 0;
  asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
  if (flags[1]) {
    // the ring is idle now (every copy landed and was consumed): chunk
    // weights f_c and l_c f_c there
    float* cf = reinterpret_cast<float*>(ring);
    float* cl = cf + nc;
    for (int hh = c; hh < QG; hh += nc) {
      const float* base = p.part + (size_t)(h0 + hh) * nc * (HS + 2);
      constexpr int kPre = 40;
      float pre[kPre];
      if (tid < HS) {
#pragma unroll
        for (int u = 0; u < kPre; u++) pre[u] = u < nc ? __ldcg(base + (size_t)u * (HS + 2) + tid) : 0.f;
      }
      float mloc = -INFINITY;
      for (int u = tid; u < nc; u += NC) {
        const float mc = __ldcg(base + (size_t)u * (HS + 2) + HS);
        cf[u] = mc;
        cl[u] = __ldcg(base + (size_t)u * (HS + 2) + HS + 1);
        mloc = fmaxf(mloc, mc);
      }
      mloc = warp_max(mloc);
      if (lane == 0) bred[warp] = mloc;
      asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
      float M = bred[0];
#pragma unroll
      for (int w = 1; w < kAttnWarps; w++) M = fmaxf(M, bred[w]);
      for (int u = tid; u < nc; u += NC) {
        const float mc = cf[u];
        const float f = mc > -INFINITY ? expf(mc - M) : 0.f;
        cf[u] = f;
        cl[u] *= f;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
      if (tid < HS) {
        float L = 0.f, acc = 0.f;
        for (int u = 0; u < nc; u++) L += cl[u];
#pragma unroll
        for (int u = 0; u < kPre; u++)
          if (u < nc) acc += pre[u] * cf[u];
        for (int u0 = kPre; u0 < nc; u0 += 8) {
          float v8[8];  // eight chunks in flight
#pragma unroll
          for (int j = 0; j < 8; j++) v8[j] = u0 + j < nc ? __ldcg(base + (size_t)(u0 + j) * (HS + 2) + tid) : 0.f;
#pragma unroll
          for (int j = 0; j < 8; j++)
            if (u0 + j < nc) acc += v8[j] * cf[u0 + j];
        }
        p.out[(size_t)(h0 + hh) * HS + tid] = L > 0.f ? acc * (1.0f / L) : 0.f;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
    }
  }
  if (tid == 0 && atomicAdd(&p.cnt[2 * kh + 1], 1u) == (unsigned)(nmerge - 1)) {
    p.cnt[2 * kh] = 0u;
    p.cnt[2 * kh + 1] = 0u;
  }
}

// RoPE frequencies (rope_neox, gguf_run.c:171): freq[j] = powf(base, -2j/hs)
__global__ void dec_rope_freq(float* freq, int hs, float base) {
  const int j = threadIdx.x;
  if (j < hs / 2) freq[j] = powf(base, -2.0f * j / hs);
}

// the chunks' states merged; out = acc / l (kv_softmax_finish, kvstore.h:99-101).
// One CTA of kCombThreads per q head, thread t on dimension t mod hs of
// chunk group t / hs (kCombThreads / hs groups, group q taking chunks q,
// q + groups, ...).  Every load that does not depend on the maximum (the
// chunk maxima and sums, and the first kCombPre accumulator values of the
// thread's chunks) is issued at once; then M = max m_c, the chunk weights
// f_c = exp(m_c - M) into shared memory, L = sum l_c f_c (a fixed-order
// block reduction) and the weighted accumulator sums, the groups added in
// group order.  Dynamic shared memory: nchunk + kCombThreads floats.
constexpr int kCombPre = 40;
__global__ void __launch_bounds__(kCombThreads) dec_attn_combine(const __grid_constant__ AttnParams p, float* out) {
  pdl_launch_dependents();  // the next kernel may take SMs now; it waits in its own prologue
  pdl_wait();  // inputs written by the previous kernel on the stream
  extern __shared__ float comb_sh[];
  __shared__ float red[32];
  const int h = blockIdx.x, t = threadIdx.x, hs = p.hs, nc = p.nchunk;
  const size_t st = (size_t)hs + 2;
  const float* base = p.part + (size_t)h * nc * st;
  float* cf = comb_sh;       // [nc] chunk weights exp(m_c - M)
  float* gs = comb_sh + nc;  // [groups][hs] group sums
  const int ng = kCombThreads / hs, g = t / hs, e = t - g * hs;
  float pre[kCombPre];
#pragma unroll
  for (int u = 0; u < kCombPre; u++) {
    const int c = g + u * ng;
    pre[u] = c < nc ? __ldcg(base + (size_t)c * st + e) : 0.f;
  }
  float m = -INFINITY;
  for (int c = t; c < nc; c += kCombThreads) m = fmaxf(m, __ldcg(base + (size_t)c * st + hs));
  m = warp_max(m);
  if ((t & 31) == 0) red[t >> 5] = m;
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kCombThreads / 32; w++) M = fmaxf(M, red[w]);
  float L = 0.f;
  for (int c = t; c < nc; c += kCombThreads) {
    const float mc = __ldcg(base + (size_t)c * st + hs);
    const float f = mc > -INFINITY ? expf(mc - M) : 0.f;
    cf[c] = f;
    L += __ldcg(base + (size_t)c * st + hs + 1) * f;
  }
  L = block_sum(L, red);  // its barriers also publish cf
  float a = 0.f;
#pragma unroll
  for (int u = 0; u < kCombPre; u++) {
    const int c = g + u * ng;
    if (c < nc) a += pre[u] * cf[c];
  }
  for (int c = g + kCombPre * ng; c < nc; c += ng) a += __ldcg(base + (size_t)c * st + e) * cf[c];
  gs[g * hs + e] = a;
  __syncthreads();
  if (t < hs) {
    float acc = 0.f;
    for (int q = 0; q < ng; q++) acc += gs[q * hs + t];
    out[(size_t)h * hs + t] = L > 0.f ? acc * (1.0f / L) : 0.f;
  }
}

// greedy argmax (gguf_run.c:253): strict '>' from index 0, so the lowest id
// wins ties and a NaN never wins
// Spread over the SMs: CTA b reduces a contiguous slice to its (value,
// index) under (value desc, index asc), NaN never winning; the last CTA to
// finish (an arrival count, put back to zero) reduces the slices' winners
// in slice order.  scratch: [kArgmaxMaxCtas] values, [kArgmaxMaxCtas]
// indices, one counter.
constexpr int kArgmaxThreads = 256, kArgmaxMaxCtas = 256;
VDEV void amax_take(float& bv, int& bi, float ov, int oi) {
  if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
    bv = ov;
    bi = oi;
  }
}
__global__ void __launch_bounds__(kArgmaxThreads) dec_argmax(const float* v, int n, int32_t* out, float* sv) {
  pdl_launch_dependents();  // the next kernel may take SMs now; it waits in its own prologue
  pdl_wait();  // inputs written by the previous kernel on the stream
  __shared__ float bv_s[32];
  __shared__ int bi_s[32];
  __shared__ int last;
  int* si = reinterpret_cast<int*>(sv + kArgmaxMaxCtas);
  unsigned int* cnt = reinterpret_cast<unsigned int*>(si + kArgmaxMaxCtas);
  const int span = (n + gridDim.x - 1) / gridDim.x, lo = blockIdx.x * span, hi = min(n, lo + span);
  float bv = -INFINITY;
  int bi = -1;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float x = __ldcg(v + i);
    if (x > bv || (bi < 0 && x == bv)) {
      bv = x;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax_take(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bv_s[warp] = bv;
    bi_s[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -INFINITY;
    int ix = -1;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) amax_take(b, ix, bv_s[w], bi_s[w]);
    sv[blockIdx.x] = b;
    si[blockIdx.x] = ix;
    __threadfence();
    last = atomicAdd(cnt, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  bv = -INFINITY;
  bi = -1;
  for (int j = threadIdx.x; j < (int)gridDim.x; j += blockDim.x) amax_take(bv, bi, __ldcg(sv + j), __ldcg(si + j));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax_take(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  __syncthreads();
  if (lane == 0) {
    bv_s[warp] = bv;
    bi_s[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -INFINITY;
    int ix = -1;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) amax_take(b, ix, bv_s[w], bi_s[w]);
    // the reference starts from v[0]: when v[0] is NaN nothing beats it
    *out = (ix < 0 || isnan(__ldcg(v))) ? 0 : ix;
    *cnt = 0u;
  }
}

// Launch with programmatic stream serialization: the kernel may be scheduled
// while the previous kernel on the stream runs and waits for it in its
// prologue (griddepcontrol.wait), so the launch latency overlaps work.
template <typename... KArgs, typename... Args>
static int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

template <class KT, int HS>
static int launch_attn_h(const AttnParams& at, int qg, int nchunk, int nkv, cudaStream_t s) {
  const dim3 grid(nchunk, nkv);
  switch (qg) {
    case 1: return launch_pdl(dec_attn_partial<KT, 1, HS, 1>, grid, dim3(kAttnChunk), 0, s, at);
    case 2: return launch_pdl(dec_attn_partial<KT, 2, HS, 2>, grid, dim3(2 * kAttnChunk), 0, s, at);
    case 4: return launch_pdl(dec_attn_partial<KT, 4, HS, 2>, grid, dim3(2 * kAttnChunk), 0, s, at);
    case 8: return launch_pdl(dec_attn_partial<KT, 8, HS, 2>, grid, dim3(2 * kAttnChunk), 0, s, at);
    default: return VIREO_ERR_UNSUPPORTED;
  }
}

template <class KT>
static int launch_attn_t(const AttnParams& at, int qg, int nchunk, int nkv, cudaStream_t s) {
  switch (at.hs) {
    case 64: return launch_attn_h<KT, 64>(at, qg, nchunk, nkv, s);
    case 128: return launch_attn_h<KT, 128>(at, qg, nchunk, nkv, s);
    default: return VIREO_ERR_UNSUPPORTED;
  }
}

static int launch_attn(const AttnParams& at, int qg, int f16, int nchunk, int nkv, cudaStream_t s) {
  return f16 ? launch_attn_t<__half>(at, qg, nchunk, nkv, s) : launch_attn_t<float>(at, qg, nchunk, nkv, s);
}

template <class KT, int HS>
static const void* attn_kernel_h(int qg) {
  switch (qg) {
    case 1: return reinterpret_cast<const void*>(&dec_attn_partial<KT, 1, HS, 1>);
    case 2: return reinterpret_cast<const void*>(&dec_attn_partial<KT, 2, HS, 2>);
    case 4: return reinterpret_cast<const void*>(&dec_attn_partial<KT, 4, HS, 2>);
    case 8: return reinterpret_cast<const void*>(&dec_attn_partial<KT, 8, HS, 2>);
    default: return nullptr;
  }
}

// the attention kernel a decoder of this shape launches
static const void* attn_kernel(int qg, int f16, int hs) {
  if (hs == 64) return f16 ? attn_kernel_h<__half, 64>(qg) : attn_kernel_h<float, 64>(qg);
  if (hs == 128) return f16 ? attn_kernel_h<__half, 128>(qg) : attn_kernel_h<float, 128>(qg);
  return nullptr;
}

// the tensor-core attention kernel (f16 cache) and its shared memory
template <int HS>
static const void* attn_mma_kernel_h(int qg, size_t* smem) {
  switch (qg) {
    case 1: *smem = attn_mma_smem<1, HS>(); return reinterpret_cast<const void*>(&dec_attn_mma<1, HS>);
    case 2: *smem = attn_mma_smem<2, HS>(); return reinterpret_cast<const void*>(&dec_attn_mma<2, HS>);
    case 4: *smem = attn_mma_smem<4, HS>(); return reinterpret_cast<const void*>(&dec_attn_mma<4, HS>);
    case 8: *smem = attn_mma_smem<8, HS>(); return reinterpret_cast<const void*>(&dec_attn_mma<8, HS>);
    default: return nullptr;
  }
}
static const void* attn_mma_kernel(int qg, int hs, size_t* smem) {
  if (hs == 64) return attn_mma_kernel_h<64>(qg, smem);
  if (hs == 128) return attn_mma_kernel_h<128>(qg, smem);
  return nullptr;
}

// positions per attention CTA: whole tiles, as few as keep about one CTA per
// SM busy over the kv heads
static int attn_mma_chunk(int npos, int nkv, int num_sms) {
  const int tiles = (npos + kAttnTile - 1) / kAttnTile;
  const int target = std::max(1, (num_sms + nkv - 1) / nkv);
  return kAttnTile * ((tiles + target - 1) / target);
}

// Every kernel of the decode chain asks for the largest shared-memory
// configuration, the one the mat-vec and MoE kernels need: an SM only holds
// CTAs of kernels that agree on it, and a programmatic launch overlaps its
// predecessor only where their CTAs can share SMs.
static int set_chain_carveout(int qg, int f16, int hs) {
  const void* fns[] = {reinterpret_cast<const void*>(&dec_rmsnorm), reinterpret_cast<const void*>(&dec_attn_combine),
                       reinterpret_cast<const void*>(&dec_argmax), attn_kernel(qg, 0, hs)};
  for (const void* fn : fns) {
    if (!fn) return VIREO_ERR_UNSUPPORTED;
    const int st = cuda_status(
        cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared));
    if (st) return st;
  }
  if (f16) {
    size_t smem = 0;
    const void* fn = attn_mma_kernel(qg, hs, &smem);
    if (!fn) return VIREO_ERR_UNSUPPORTED;
    int st = cuda_status(
        cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared));
    if (!st) st = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (st) return st;
  }
  return VIREO_OK;
}

}  // namespace vireo

using namespace vireo;

struct gguf_decoder {
  gguf_decoder_desc d;
  std::vector<gguf_decoder_layer> L;
  std::vector<void*> wqkv;  // per layer: wq | wk | wv rows in one buffer (one mat-vec), or null
  float* freq = nullptr;
  Ctx* c = nullptr;
  float *x = nullptr, *xb = nullptr, *y = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr,
        *part = nullptr, *logits = nullptr;
  void *kc = nullptr, *vc = nullptr;
  size_t layer_kv = 0;  // elements of one layer's K (or V) cache
  int max_chunk = 0;
  unsigned int* attn_cnt = nullptr;  // [n_kv_heads][2] merge counters of the tensor-core attention
  float* amax = nullptr;             // argmax scratch: per-CTA winners and the arrival count
};

extern "C" {

void gguf_decoder_destroy(gguf_decoder* dec) {
  if (!dec) return;
  for (void* p : {(void*)dec->x, (void*)dec->xb, (void*)dec->y, (void*)dec->q, (void*)dec->att, (void*)dec->part,
                  (void*)dec->logits, dec->kc, dec->vc, (void*)dec->freq, (void*)dec->attn_cnt, (void*)dec->amax})
    if (p) cudaFree(p);
  for (void* p : dec->wqkv)
    if (p) cudaFree(p);
  delete dec;
}

int gguf_decoder_create(const gguf_decoder_desc* desc, const gguf_decoder_layer* layers, gguf_decoder** out) {
  if (!desc || !layers || !out) return VIREO_ERR_ARG;
  *out = nullptr;
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) return st;
  const gguf_decoder_desc& D = *desc;
  if (D.n_layers < 1 || D.dim < 1 || D.dim > 16384 || D.n_heads < 1 || D.n_kv_heads < 1 ||
      D.n_heads % D.n_kv_heads || (D.head_size != 64 && D.head_size != 128) ||
      (D.n_heads / D.n_kv_heads != 1 && D.n_heads / D.n_kv_heads != 2 && D.n_heads / D.n_kv_heads != 4 &&
       D.n_heads / D.n_kv_heads != 8) ||
      (size_t)(D.n_heads + 2 * D.n_kv_heads) * D.head_size * 4 > 48 * 1024 ||
      D.vocab < 1 || D.max_ctx < 1 || D.max_ctx > kMaxCtx || !D.tok_embd || !D.out_norm || !D.lm_head)
    return VIREO_ERR_ARG;
  int be, bb;
  if (type_block(D.tok_embd_type, &be, &bb) || D.dim % be || type_block(D.lm_head_type, &be, &bb) || D.dim % be)
    return VIREO_ERR_UNSUPPORTED;
  const int nq = D.n_heads * D.head_size, nk = D.n_kv_heads * D.head_size;
  for (int l = 0; l < D.n_layers; l++) {
    const gguf_decoder_layer& y = layers[l];
    if (!y.attn_norm || !y.ffn_norm || !y.wq || !y.wk || !y.wv || !y.wo || !y.moe) return VIREO_ERR_ARG;
    if ((y.q_norm && y.q_norm_len != D.head_size && y.q_norm_len != nq) ||
        (y.k_norm && y.k_norm_len != D.head_size && y.k_norm_len != nk))
      return VIREO_ERR_ARG;
    for (uint32_t t : {y.wq_type, y.wk_type, y.wv_type})
      if (type_block(t, &be, &bb) || D.dim % be) return VIREO_ERR_UNSUPPORTED;
    if (type_block(y.wo_type, &be, &bb) || nq % be) return VIREO_ERR_UNSUPPORTED;
    // the MoE block reads hb and writes x over its own dim: it must be D.dim
    MoeView mv;
    if (moe_view(y.moe, &mv) || !mv.desc || mv.desc->dim != D.dim) return VIREO_ERR_ARG;
  }
  if ((st = set_chain_carveout(D.n_heads / D.n_kv_heads, D.kv_f16, D.head_size))) return st;
  gguf_decoder* dec = new gguf_decoder();
  dec->d = D;
  dec->L.assign(layers, layers + D.n_layers);
  dec->c = c;
  // chunks per head: the chunk-parallel kernel's, or the tensor-core one's,
  // which is at most the tiles of the longest context and at most its CTA
  // target per kv head (not monotone in the context length, so bounded by both)
  dec->max_chunk = std::max((D.max_ctx + kAttnChunk - 1) / kAttnChunk,
                            std::min((D.max_ctx + kAttnTile - 1) / kAttnTile,
                                     std::max(1, (c->num_sms + D.n_kv_heads - 1) / D.n_kv_heads)));
  dec->layer_kv = (size_t)D.n_kv_heads * D.max_ctx * D.head_size;
  const size_t kvb = dec->layer_kv * D.n_layers * (D.kv_f16 ? 2 : 4);
  if ((st = cuda_status(cudaMalloc(&dec->x, (size_t)D.dim * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->xb, (size_t)D.dim * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->y, (size_t)D.dim * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->q, (size_t)(nq + 2 * nk) * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->freq, (size_t)D.head_size / 2 * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->att, (size_t)nq * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->part, (size_t)D.n_heads * dec->max_chunk * (D.head_size + 2) * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->logits, (size_t)D.vocab * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->attn_cnt, (size_t)D.n_kv_heads * 2 * 4))) ||
      (st = cuda_status(cudaMemset(dec->attn_cnt, 0, (size_t)D.n_kv_heads * 2 * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->amax, (size_t)(2 * kArgmaxMaxCtas + 1) * 4))) ||
      (st = cuda_status(cudaMemset(dec->amax, 0, (size_t)(2 * kArgmaxMaxCtas + 1) * 4))) ||
      (st = cuda_status(cudaMalloc(&dec->kc, kvb))) || (st = cuda_status(cudaMalloc(&dec->vc, kvb))) ||
      (st = cuda_status(cudaMemset(dec->x, 0, (size_t)D.dim * 4)))) {
    gguf_decoder_destroy(dec);
    return st;
  }
  // q, k and v are one vector: one mat-vec over wq | wk | wv writes all three
  dec->k = dec->q + nq;
  dec->v = dec->k + nk;
  dec_rope_freq<<<1, 128, 0, c->stream>>>(dec->freq, D.head_size, D.rope_base);
  dec->wqkv.assign(D.n_layers, nullptr);
  for (int l = 0; l < D.n_layers; l++) {
    const gguf_decoder_layer& y = layers[l];
    if (y.wq_type != y.wk_type || y.wq_type != y.wv_type) continue;
    const size_t rb = row_bytes(y.wq_type, D.dim);
    void* w = nullptr;
    if ((st = cuda_status(cudaMalloc(&w, rb * (nq + 2 * nk)))) ||
        (st = cuda_status(cudaMemcpyAsync(w, y.wq, rb * nq, cudaMemcpyDeviceToDevice, c->stream))) ||
        (st = cuda_status(cudaMemcpyAsync((uint8_t*)w + rb * nq, y.wk, rb * nk, cudaMemcpyDeviceToDevice, c->stream))) ||
        (st = cuda_status(
             cudaMemcpyAsync((uint8_t*)w + rb * (nq + nk), y.wv, rb * nk, cudaMemcpyDeviceToDevice, c->stream)))) {
      if (w) cudaFree(w);
      gguf_decoder_destroy(dec);
      return st;
    }
    dec->wqkv[l] = w;
  }
  if ((st = cuda_status(cudaStreamSynchronize(c->stream)))) {
    gguf_decoder_destroy(dec);
    return st;
  }
  *out = dec;
  return VIREO_OK;
}

// one step; the token is a host value (token_dev NULL) or read on the device
static int decoder_step(gguf_decoder* dec, int token, const int32_t* token_dev, int pos, float* logits, int32_t* next,
                        void* stream) {
  if (!dec) return VIREO_ERR_ARG;
  const gguf_decoder_desc& D = dec->d;
  if ((!token_dev && (token < 0 || token >= D.vocab)) || pos < 0 || pos >= D.max_ctx) return VIREO_ERR_ARG;
  cudaStream_t s = stream ? (cudaStream_t)stream : dec->c->stream;
  Ctx* c = dec->c;
  const int d = D.dim, hs = D.head_size, nq = D.n_heads * hs, nk = D.n_kv_heads * hs;
  int st;
  // embedding row (gguf_run.c:218)
  if (token_dev)
    st = launch_embed(D.tok_embd_type, D.tok_embd, token_dev, D.vocab, dec->x, d, c->d_err, s);
  else
    st = launch_dequant(D.tok_embd_type, (const uint8_t*)D.tok_embd + (size_t)token * row_bytes(D.tok_embd_type, d),
                        dec->x, d, s);
  if (st) return st;
  const int npos = pos + 1, nchunk = (npos + kAttnChunk - 1) / kAttnChunk;
  const size_t kv_el = D.kv_f16 ? 2 : 4;
  for (int l = 0; l < D.n_layers; l++) {
    const gguf_decoder_layer& y = dec->L[l];
    // xb = attn_norm(x); q | k | v = W . xb   (gguf_run.c:222-225): one
    // mat-vec whose CTAs normalise x themselves when wq, wk, wv share a type
    st = dec->wqkv[l] ? gemv_dev_fast(c, y.wq_type, dec->wqkv[l], dec->x, dec->q, d, nq + 2 * nk, s, y.attn_norm,
                                      D.eps, kDecPrefetch)
                      : VIREO_ERR_UNSUPPORTED;
    if (st == VIREO_ERR_UNSUPPORTED) {
      if ((st = launch_pdl(dec_rmsnorm, dim3(1), dim3(kDecThreads), 0, s, dec->x, (const float*)nullptr,
                           y.attn_norm, dec->xb, d, D.eps)))
        return st;
      if (dec->wqkv[l]) {
        if ((st = gemv_dev(c, y.wq_type, dec->wqkv[l], dec->xb, dec->q, d, nq + 2 * nk, s))) return st;
      } else if ((st = gemv_dev(c, y.wq_type, y.wq, dec->xb, dec->q, d, nq, s)) ||
                 (st = gemv_dev(c, y.wk_type, y.wk, dec->xb, dec->k, d, nk, s)) ||
                 (st = gemv_dev(c, y.wv_type, y.wv, dec->xb, dec->v, d, nk, s))) {
        return st;
      }
    } else if (st) {
      return st;
    }
    // q/k post-processing, KV append and attention over every cached position
    AttnParams at;
    at.q = dec->q;
    at.k = dec->k;
    at.v = dec->v;
    at.bq = y.bq;
    at.bk = y.bk;
    at.bv = y.bv;
    at.qn = y.q_norm;
    at.kn = y.k_norm;
    at.qn_len = y.q_norm_len;
    at.kn_len = y.k_norm_len;
    at.freq = dec->freq;
    at.kc = (uint8_t*)dec->kc + (size_t)l * dec->layer_kv * kv_el;
    at.vc = (uint8_t*)dec->vc + (size_t)l * dec->layer_kv * kv_el;
    at.nh = D.n_heads;
    at.nkv = D.n_kv_heads;
    at.hs = hs;
    at.pos = pos;
    at.npos = npos;
    at.max_ctx = D.max_ctx;
    at.nchunk = nchunk;
    at.scale = 1.0f / sqrtf((float)hs);
    at.eps = D.eps;
    at.part = dec->part;
    at.cnt = dec->attn_cnt;
    at.out = dec->att;
    at.err = c->d_err;
    if (D.kv_f16) {
      // tensor-core attention per (chunk, kv head), the chunk merge in the same kernel
      size_t smem = 0;
      const void* fn = attn_mma_kernel(D.n_heads / D.n_kv_heads, hs, &smem);
      const int C = attn_mma_chunk(npos, D.n_kv_heads, c->num_sms);
      at.nchunk = (npos + C - 1) / C;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(at.nchunk, D.n_kv_heads);
      cfg.blockDim = dim3(kAttnMmaThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int Cv = C;
      void* args[] = {&at, &Cv};
      if ((st = cuda_status(cudaLaunchKernelExC(&cfg, fn, args)))) return st;
    } else {
      if ((st = launch_attn(at, D.n_heads / D.n_kv_heads, D.kv_f16, nchunk, D.n_kv_heads, s))) return st;
      if ((st = launch_pdl(dec_attn_combine, dim3(D.n_heads), dim3(kCombThreads),
                           (size_t)(nchunk + kCombThreads) * sizeof(float), s, at, dec->att)))
        return st;
    }
    st = gemv_dev_fast(c, y.wo_type, y.wo, dec->att, dec->y, nq, d, s, nullptr, 0.f, kDecPrefetch);
    if (st == VIREO_ERR_UNSUPPORTED) st = gemv_dev(c, y.wo_type, y.wo, dec->att, dec->y, nq, d, s);
    if (st) return st;
    // x += attention output; x += MoE(ffn_norm(x))   (gguf_run.c:237-239): the
    // residual add and the norm inside the MoE kernel
    if ((st = moe_ffn_norm(y.moe, dec->x, dec->y, y.ffn_norm, D.eps, s))) return st;
  }
  if (logits || next) {
    float* lg = logits ? logits : dec->logits;
    // logits = lm_head . out_norm(x)   (gguf_run.c:249-251), the norm inside the mat-vec where it can be
    st = gemv_dev_fast(c, D.lm_head_type, D.lm_head, dec->x, lg, d, D.vocab, s, D.out_norm, D.eps, kDecPrefetch);
    if (st == VIREO_ERR_UNSUPPORTED) {
      if ((st = launch_pdl(dec_rmsnorm, dim3(1), dim3(kDecThreads), 0, s, dec->x, (const float*)nullptr,
                           D.out_norm, dec->xb, d, D.eps)))
        return st;
      st = gemv_dev(c, D.lm_head_type, D.lm_head, dec->xb, lg, d, D.vocab, s);
    }
    if (st) return st;
    if (next && (st = launch_pdl(dec_argmax, dim3(std::min(std::min(c->num_sms, kArgmaxMaxCtas), (D.vocab + 1023) / 1024)),
                                 dim3(kArgmaxThreads), 0, s, (const float*)lg, D.vocab, next, dec->amax)))
      return st;
  }
  return cuda_status(cudaGetLastError());
}

int gguf_decoder_step(gguf_decoder* dec, int token, int pos, float* logits, int32_t* next, void* stream) {
  return decoder_step(dec, token, nullptr, pos, logits, next, stream);
}

int gguf_decoder_step_dev(gguf_decoder* dec, const int32_t* token, int pos, float* logits, int32_t* next,
                          void* stream) {
  if (!token) return VIREO_ERR_ARG;
  return decoder_step(dec, 0, token, pos, logits, next, stream);
}

const float* gguf_decoder_hidden(const gguf_decoder* dec) { return dec ? dec->x : nullptr; }

int gguf_decoder_sync(gguf_decoder* dec, void* stream) {
  if (!dec) return VIREO_ERR_ARG;
  cudaStream_t s = stream ? (cudaStream_t)stream : dec->c->stream;
  int st = cuda_status(cudaStreamSynchronize(s));
  if (st) return st;
  int herr = 0;
  if ((st = cuda_status(cudaMemcpy(&herr, dec->c->d_err, sizeof(int), cudaMemcpyDeviceToHost)))) return st;
  if (herr) {
    cudaMemset(dec->c->d_err, 0, sizeof(int));
    cudaMemset(dec->attn_cnt, 0, (size_t)dec->d.n_kv_heads * 2 * 4);  // a merge may have given up mid-count
    return herr;
  }
  for (const auto& y : dec->L)
    if ((st = gguf_moe_sync(y.moe, stream))) return st;
  return VIREO_OK;
}

}  // extern "C"
