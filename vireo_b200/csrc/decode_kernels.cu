// Decode kernels: the MoE FFN block (one token, all phases in one
// cooperative launch) and the stand-alone quantised GEMV behind
// gguf_matmul.  See moe_decode.cuh and engine.cuh for the design.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "moe_decode.cuh"
#include "vireo_internal.h"

namespace vireo {

struct Ctl {
  int abort;
  float wsum;  // renorm denominator
  int ids[kMaxTopK];
  float wts[kMaxTopK];
  int tile_cnt[2];  // down units finished per tile buffer
  float nred[kConsumerWarps];  // gemv_kernel: per-warp sums of squares for the fused norm
};

VDEV void trace(const MoeDecodeParams& p, int slot) {
  if (p.trace) p.trace[blockIdx.x * kTraceSlots + slot] = now_ns();
}

VDEV void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

VDEV bool aborted(const Ctl* c) { return *reinterpret_cast<const volatile int*>(&c->abort) != 0; }
VDEV void do_abort(Ctl* c, int* err, int code) {
  set_error(err, code);
  *reinterpret_cast<volatile int*>(&c->abort) = 1;
}

// consume_unit variant that can skip the math (inactive unit) while keeping
// the partial/counter protocol intact
template <class S>
VDEV bool consume(const uint8_t* stage, const StageGeom& sg, int v, int nseg, int w, const uint8_t* btab,
                  const float* sx, float* part, int* ucnt, const LaneCtx& L, float* val, bool active, BFrag& bf) {
  return consume_unit<S>(stage, sg, v, active ? nseg : 0, kConsumerWarps, w, btab, sx, part, ucnt, L, val, bf);
}

// Warp-collective stage wait: lane 0 waits (bounded), the result and the
// completed phase are shared with the warp.  False when aborted or timed out
// (the timeout is recorded).
VDEV bool warp_wait(uint64_t* bar, uint32_t par, Ctl* ctl, int* err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    ok = (!aborted(ctl) && mbar_wait(bar, par, &ctl->abort)) ? 1 : 0;
    if (!ok && !aborted(ctl)) do_abort(ctl, err, VIREO_ERR_TIMEOUT);
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

// ---------------------------------------------------------------------------
// MoE decode kernel
// ---------------------------------------------------------------------------

// Cooperative (block-wide among nthr threads starting at thread 0) load of
// n floats from global into shared memory with 16-byte loads.
VDEV void stage_vec(const float* g, float* s, int n, int tid, int nthr, bool bypass_l1) {
  const float4* g4 = reinterpret_cast<const float4*>(g);
  float4* s4 = reinterpret_cast<float4*>(s);
  for (int i = tid; i < n / 4; i += nthr) s4[i] = bypass_l1 ? __ldcg(g4 + i) : __ldg(g4 + i);
}

// As stage_vec with L2-only loads (data other CTAs wrote) and 8 loads in
// flight per thread.
VDEV void stage_vec_cg8(const float* g, float* s, int n, int tid, int nthr) {
  const float4* g4 = reinterpret_cast<const float4*>(g);
  float4* s4 = reinterpret_cast<float4*>(s);
  const int n4 = n / 4;
  for (int i0 = tid; i0 < n4; i0 += 8 * nthr) {
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (i0 + j * nthr < n4) v[j] = __ldcg(g4 + i0 + j * nthr);
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (i0 + j * nthr < n4) s4[i0 + j * nthr] = v[j];
  }
}

// The decode kernel body.  ROUTED: the route comes from the caller (rt) and
// the router phase is skipped; otherwise every CTA computes it.
template <class SG, class SD, bool ROUTED>
__device__ __forceinline__ void moe_decode_body(const MoeDecodeParams& p, const MoeRoute* rt) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kDecodeThreads / 32 + 1];
  // gate/up ring (S stages) and down ring (SD slots over the same memory)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* full_d = empty + kMaxStages;
  uint64_t* empty_d = full_d + kMaxStages;
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
  float* part = reinterpret_cast<float*>(smem + p.off_part);
  float* part_d = reinterpret_cast<float*>(smem + p.off_part_d);
  int* ucnt = reinterpret_cast<int*>(smem + p.off_ucnt);
  int* ucnt_d = ucnt + kMaxStages;
  float* ytile = reinterpret_cast<float*>(smem + p.off_ytile); // [2][k][16] expert rows of a tile
  uint8_t* xtab = smem + p.off_xtab;
  float* xsx = reinterpret_cast<float*>(smem + p.off_xsx);
  uint8_t* htab = smem + p.off_htab;
  float* hsx = reinterpret_cast<float*>(smem + p.off_hsx);
  float* stg = reinterpret_cast<float*>(smem + p.off_stg);  // x staging
  uint8_t* stages = smem + p.off_stage;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = kConsumerWarps;
  constexpr int NC = W * 32;  // consumer threads
  const int G = gridDim.x, cta = blockIdx.x;
  const int d = p.d, fe = p.fe, ne = p.ne, k = p.k, S = p.nstages, SD_ = p.nstages_d;
  MoeSync* sy = p.s.sync;

  if (threadIdx.x == 0) {
    trace(p, kTrStart);
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], kProducerThreads);  // every producer's copies
      mbar_init(&empty[s], W);
    }
    for (int s = 0; s < SD_; s++) {
      mbar_init(&full_d[s], kProducerThreads);
      mbar_init(&empty_d[s], W);
    }
    ctl->abort = 0;
    ctl->tile_cnt[0] = ctl->tile_cnt[1] = 0;
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < 2 * kMaxStages; i += blockDim.x) ucnt[i] = 0;
  // the next token's kernel may start its own prologue as SMs free up
  pdl_launch_dependents();

  if constexpr (ROUTED) {
    // ---- caller's route: x tables and the selection, no router phase --------
    pdl_wait();
    stage_vec(p.hb, stg, d, threadIdx.x, blockDim.x, false);
    if (threadIdx.x < k) {
      ctl->ids[threadIdx.x] = rt->ids[threadIdx.x];
      ctl->wts[threadIdx.x] = rt->wts[threadIdx.x];
      if (cta == 0) {
        if (p.ids_out) p.ids_out[threadIdx.x] = rt->ids[threadIdx.x];
        if (p.wts_out) p.wts_out[threadIdx.x] = rt->wts[threadIdx.x];
      }
    }
    __syncthreads();
    build_tables<SG>(stg, xtab, xsx, d / kSegElems, warp, (int)(blockDim.x / 32), lane);
    __syncthreads();
    if (threadIdx.x == 0) trace(p, kTrRouted);
  } else {
  // ---- phase R: router partial dot products --------------------------------
  // Router rows are weights (independent of the previous kernel): their loads
  // are issued before waiting on the previous kernel in the stream.
  {
    const int nchunk = d / kRouterChunk;
    const int ntask = ne * nchunk, nw = G * (int)(blockDim.x / 32);
    const int gw = warp * G + cta;  // spread tasks over all CTAs first
    float4 r0[4], r1[4];
    const bool has0 = gw < ntask, has1 = gw + nw < ntask;
    if (has0) {
      const int e = gw / nchunk, c = gw - e * nchunk;
      const float4* row = reinterpret_cast<const float4*>(p.router + (size_t)e * d + (size_t)c * kRouterChunk);
#pragma unroll
      for (int i = 0; i < 4; i++) r0[i] = __ldg(row + lane + 32 * i);
    }
    if (has1) {
      const int t1 = gw + nw, e = t1 / nchunk, c = t1 - e * nchunk;
      const float4* row = reinterpret_cast<const float4*>(p.router + (size_t)e * d + (size_t)c * kRouterChunk);
#pragma unroll
      for (int i = 0; i < 4; i++) r1[i] = __ldg(row + lane + 32 * i);
    }
    pdl_wait();
    stage_vec(p.hb, stg, d, threadIdx.x, blockDim.x, false);
    for (int task = gw, it = 0; task < ntask; task += nw, it++) {
      const int e = task / nchunk, c = task - e * nchunk;
      float4 r[4];
      if (it == 0) {
#pragma unroll
        for (int i = 0; i < 4; i++) r[i] = r0[i];
      } else if (it == 1) {
#pragma unroll
        for (int i = 0; i < 4; i++) r[i] = r1[i];
      } else {
        const float4* row = reinterpret_cast<const float4*>(p.router + (size_t)e * d + (size_t)c * kRouterChunk);
#pragma unroll
        for (int i = 0; i < 4; i++) r[i] = __ldg(row + lane + 32 * i);
      }
      const float4* xv = reinterpret_cast<const float4*>(p.hb + (size_t)c * kRouterChunk);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 xx = __ldg(xv + lane + 32 * i);
        s = fmaf(r[i].x, xx.x, s);
        s = fmaf(r[i].y, xx.y, s);
        s = fmaf(r[i].z, xx.z, s);
        s = fmaf(r[i].w, xx.w, s);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) p.s.logit_part[(size_t)c * ne + e] = s;
    }
    __syncthreads();
    // every CTA has written its router partials once router_arrive == G
    if (threadIdx.x == 0) {
      trace(p, kTrRouterDone);
      red_add_release_gpu(&sy->router_arrive.v, 1u);
    }
    // x table while the other CTAs finish their router partials
    build_tables<SG>(stg, xtab, xsx, d / kSegElems, warp, (int)(blockDim.x / 32), lane);
    if (threadIdx.x == 0) {
      if (!wait_geq(&sy->router_arrive.v, (unsigned)G, p.s.err)) ctl->abort = 1;
      trace(p, kTrPartials);
    }
    __syncthreads();
    // ---- softmax + top-k in every CTA (no second hop) ----------------------
    // logits l[e] = sum of the chunk partials in chunk order; p = softmax(l);
    // expert e takes rank r = #{j : p_j > p_e, or p_j == p_e and j < e}, the
    // position the reference's greedy strict-'>' selection gives it
    // (gguf_run.c:190-191); ranks < k are the selection.  NaN never ranks.
    float* pr = reinterpret_cast<float*>(htab);  // probabilities (htab idle until the down phase)
    if (!aborted(ctl)) {
      float lv = -INFINITY;
      const int e = threadIdx.x;
      if (e < ne) {
        float part_c[8];
#pragma unroll
        for (int c = 0; c < 8; c++) part_c[c] = (c < nchunk) ? __ldcg(p.s.logit_part + (size_t)c * ne + e) : 0.f;
        lv = 0.f;
#pragma unroll
        for (int c = 0; c < 8; c++)
          if (c < nchunk) lv += part_c[c];
      }
      float m = lv;
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) red[warp] = m;
      __syncthreads();
      float mx = -INFINITY;
      for (int i = 0; i < (int)(blockDim.x / 32); i++) mx = fmaxf(mx, red[i]);
      const float ex = (e < ne) ? expf(lv - mx) : 0.f;
      float sm = ex;
#pragma unroll
      for (int o = 16; o; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
      __syncthreads();
      if (lane == 0) red[warp] = sm;
      __syncthreads();
      float sum = 0.f;
      for (int i = 0; i < (int)(blockDim.x / 32); i++) sum += red[i];
      const float pe = ex / sum;
      if (e < ne) pr[e] = pe;
      __syncthreads();
      if (e < ne && !isnan(pe)) {
        int rank = 0;
        const float4* pr4 = reinterpret_cast<const float4*>(pr);
#pragma unroll 4
        for (int j4 = 0; j4 < ne / 4; j4++) {
          const float4 q = pr4[j4];
          const int j = 4 * j4;
          rank += (q.x > pe) || (q.x == pe && j < e);
          rank += (q.y > pe) || (q.y == pe && j + 1 < e);
          rank += (q.z > pe) || (q.z == pe && j + 2 < e);
          rank += (q.w > pe) || (q.w == pe && j + 3 < e);
        }
        for (int j = ne & ~3; j < ne; j++) {
          const float pj = pr[j];
          rank += (pj > pe) || (pj == pe && j < e);
        }
        if (rank < k) {
          ctl->ids[rank] = e;
          ctl->wts[rank] = pe;
        }
      }
      // fewer than k selectable experts (NaN probabilities): unused slots
      // hold id -1, weight -1 as in the reference's scan
      const int nsel = __syncthreads_count(e < ne && !isnan(pe));
      const int t = threadIdx.x;
      if (t < k && t >= nsel) {
        ctl->ids[t] = -1;
        ctl->wts[t] = -1.f;
      }
      __syncthreads();
      if (t == 0) {
        // renorm denominator: the sequential rank-order sum (gguf_run.c:192)
        float ws = 0.f;
#pragma unroll 1
        for (int j = 0; j < k; j++) ws = ws + ctl->wts[j];
        ctl->wsum = ws;
      }
      __syncthreads();
      if (t < k) {
        const float ws = ctl->wsum;
        float w = ctl->wts[t];
        if (p.renorm && ws > 0.f) w = w / ws;
        ctl->wts[t] = w;
        if (cta == 0) {
          if (p.ids_out) p.ids_out[t] = ctl->ids[t];
          if (p.wts_out) p.wts_out[t] = w;
        }
      }
      if (t == 0) trace(p, kTrRouted);
    }
    __syncthreads();
  }
  }

  // device address of slice `which` (0 gate, 1 up, 2 down) of expert slot t
  auto expert_ptr = [&](int t, int which) -> const uint8_t* {
    if constexpr (ROUTED) {
      return ctl->ids[t] < 0 ? nullptr : rt->ptr[t][which];
    } else {
      const int e = ctl->ids[t];
      return e < 0 ? nullptr : p.exp_tab[3 * e + which];
    }
  };

  const int rgG = fe / 8, UG = k * rgG, ntile = d / 16;
  const int g0 = (int)((long long)cta * UG / G), g1 = (int)((long long)(cta + 1) * UG / G);
  const int my_tiles = (cta < ntile) ? (ntile - 1 - cta) / G + 1 : 0;

  const int nG = g1 - g0, nD = my_tiles * k;
  if (warp >= W) {
    // ---- producers: 16-byte cp.async copies ---------------------------------
    const int ptid = threadIdx.x - NC;
    // gate/up units: a contiguous range per CTA
    if (ptid == 0) trace(p, kTrProdFirst);
    for (int v = 0; v < nG; v++) {
      const int slot = v % S;
      if (!warp_wait(&empty[slot], ((uint32_t)(v / S) & 1u) ^ 1u, ctl, p.s.err)) break;
      const int u = g0 + v, t = u / rgG, rg = u - t * rgG;
      const uint8_t* gb = expert_ptr(t, 0);
      const uint8_t* ub = expert_ptr(t, 1);
      const uint8_t* gsrc = gb ? gb + (size_t)(8 * rg) * p.sg_gu.rb : nullptr;
      const uint8_t* usrc = ub ? ub + (size_t)(8 * rg) * p.sg_gu.rb : nullptr;
      issue_unit(stages + (size_t)slot * p.stage_bytes, &full[slot], gsrc, usrc, p.sg_gu, ptid, kProducerThreads);
    }
    // down units: every expert slot of each of this CTA's 16-row tiles, in
    // the down ring.  A slot's first use waits for the last release of every
    // gate/up stage it overlaps (the down weights do not depend on h, so
    // they stream in while gate/up is still being consumed).
    if (ptid == 0) trace(p, kTrProdFirstD);
    for (int j = 0; j < nD && !aborted(ctl); j++) {
      const int slot = j % SD_;
      bool ok = true;
      if (j < SD_) {
        const uint32_t lo = (uint32_t)slot * p.dslot_bytes, hi = lo + p.dslot_bytes - 1u;
        for (int st = (int)(lo / p.stage_bytes); ok && st <= (int)(hi / p.stage_bytes) && st < nG; st++)
          ok = warp_wait(&empty[st], (uint32_t)((nG - 1 - st) / S) & 1u, ctl, p.s.err);
      } else {
        ok = warp_wait(&empty_d[slot], ((uint32_t)(j / SD_) & 1u) ^ 1u, ctl, p.s.err);
      }
      if (!ok) break;
      const int i = j / k, t = j - i * k, tile = cta + i * G;
      const uint8_t* db = expert_ptr(t, 2);
      const uint8_t* src = db ? db + (size_t)(16 * tile) * p.sg_d.rb : nullptr;
      issue_unit(stages + (size_t)slot * p.dslot_bytes, &full_d[slot], src, src ? src + 8 * (size_t)p.sg_d.rb : nullptr,
                 p.sg_d, ptid, kProducerThreads);
    }
    if (ptid == 0) trace(p, kTrProdLast);
    cp_async_wait_all();  // no copy may still target this CTA's shared memory at exit
    if (ptid == 0) trace(p, kTrProdDrained);
    return;
  }

  // ---- consumers -------------------------------------------------------------
  const LaneCtx L = lane_ctx();
  BFrag bf;
  bf.reset();
  for (int v = 0; v < nG; v++) {
    const int slot = v % S;
    if (!warp_wait(&full[slot], (uint32_t)(v / S) & 1u, ctl, p.s.err)) break;
    const int u = g0 + v;
    if (threadIdx.x == 0 && v < kTrUnits) trace(p, kTrUnitBase + 2 * v);
    const int t = u / rgG, rg = u - t * rgG;
    const bool active = ctl->ids[t] >= 0;
    float val = 0.f;
    const bool last = consume<SG>(stages + (size_t)slot * p.stage_bytes, p.sg_gu, v, p.d / kSegElems, warp, xtab,
                                  xsx, part + slot * p.part_stride, &ucnt[slot], L, &val, active, bf);
    if (last) {
      const float up = __shfl_sync(0xffffffffu, val, (lane + 8) & 31);
      float hv = 0.f;
      if (active && lane < 8) {
        // the reference's SwiGLU, gguf_run.c:206
        hv = (val / (1.0f + expf(-val))) * up;
        p.s.hbuf[(size_t)t * fe + 8 * rg + lane] = hv;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (threadIdx.x == 0 && v < kTrUnits) trace(p, kTrUnitBase + 2 * v + 1);
  }
  // publish this CTA's gate/up results (h rows in scratch): one count
  named_bar(1, NC);
  if (threadIdx.x == 0) {
    trace(p, kTrGDone);
    __threadfence();
    red_add_release_gpu(&sy->g_done.v, (unsigned)(g1 - g0));
  }

  if (my_tiles > 0) {
    // ---- every h row written: build the k down-projection B tables ----------
    if (threadIdx.x == 0) {
      if (!aborted(ctl) && !wait_geq(&sy->g_done.v, (unsigned)UG, p.s.err)) ctl->abort = 1;
      trace(p, kTrGAll);
    }
    named_bar(1, NC);
    if (!aborted(ctl)) {
      if (threadIdx.x == 0) trace(p, kTrDbg + 0);
      // h rows (written by other CTAs) into the table area with coalesced
      // 16-byte loads, then the tables built in place
      stage_vec_cg8(p.s.hbuf, reinterpret_cast<float*>(htab), k * fe, threadIdx.x, NC);
      named_bar(1, NC);
      if (threadIdx.x == 0) trace(p, kTrDbg + 2);
      build_tables<SD>(reinterpret_cast<const float*>(htab), htab, hsx, k * fe / kSegElems, warp, W, lane);
      if (threadIdx.x == 0) trace(p, kTrDbg + 1);
    }
    named_bar(1, NC);
    if (threadIdx.x == 0) trace(p, kTrHtab);

    // ---- down units: tile-major, combined in this CTA ------------------------
    for (int i = 0, j = 0; i < my_tiles; i++) {
      const int tb = i & 1;
      for (int t = 0; t < k; t++, j++) {
        const int slot = j % SD_;
        const bool ok = warp_wait(&full_d[slot], (uint32_t)(j / SD_) & 1u, ctl, p.s.err);
        if (threadIdx.x == 0 && nG + j < kTrUnits) trace(p, kTrUnitBase + 2 * (nG + j));
        const int tile = cta + i * G;
        const bool active = ok && ctl->ids[t] >= 0;
        float val = 0.f;
        const bool last = consume<SD>(stages + (size_t)slot * p.dslot_bytes, p.sg_d, j, fe / kSegElems, warp,
                                      htab + (size_t)t * p.htab_bytes, hsx + (size_t)t * p.hsx_count,
                                      part_d + slot * p.part_stride, &ucnt_d[slot], L, &val, active, bf);
        if (last) {
          if (lane < 16) ytile[(tb * k + t) * 16 + lane] = active ? val : 0.f;
          __syncwarp();
          int done = 0;
          if (lane == 0) {
            __threadfence_block();
            done = (atomicAdd(&ctl->tile_cnt[tb], 1) == k - 1);
          }
          done = __shfl_sync(0xffffffffu, done, 0);
          if (done) {
            __threadfence_block();
            if (lane < 16 && ok) {
              // the reference's combine order: acc = sum over rank t of w_t * y_t, then x += acc
              const int r = 16 * tile + lane;
              float acc = 0.f;
              for (int tt = 0; tt < k; tt++)
                if (ctl->ids[tt] >= 0)
                  acc = __fadd_rn(acc, __fmul_rn(ctl->wts[tt], ((volatile float*)ytile)[(tb * k + tt) * 16 + lane]));
              p.x[r] = __fadd_rn(p.x[r], acc);
            }
            __syncwarp();
            if (lane == 0) ctl->tile_cnt[tb] = 0;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_d[slot]);
        if (threadIdx.x == 0 && nG + j < kTrUnits) trace(p, kTrUnitBase + 2 * (nG + j) + 1);
      }
    }
  }
  if (threadIdx.x == 0) trace(p, kTrDDone);

  // ---- launch exit: the last CTA out resets the per-launch words -------------
  named_bar(1, NC);
  if (threadIdx.x == 0) {
    if (atom_add_acq_rel_gpu(&sy->exit_cnt.v, 1u) == (unsigned)G - 1u) {
      sy->router_arrive.v = 0u;
      sy->g_done.v = 0u;
      __threadfence();
      sy->exit_cnt.v = 0u;
    }
  }
}

template <class SG, class SD>
__global__ void __launch_bounds__(kDecodeThreads, 1) moe_decode_kernel(const __grid_constant__ MoeDecodeParams p) {
  moe_decode_body<SG, SD, false>(p, nullptr);
}

template <class SG, class SD>
__global__ void __launch_bounds__(kDecodeThreads, 1)
    moe_routed_kernel(const __grid_constant__ MoeDecodeParams p, const __grid_constant__ MoeRoute r) {
  moe_decode_body<SG, SD, true>(p, &r);
}

// ---------------------------------------------------------------------------
// Stand-alone GEMV: y[d] = W[d x n] . x[n]  (fast formats, d % 16 == 0)
// ---------------------------------------------------------------------------
template <class SF>
__global__ void __launch_bounds__(kDecodeThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
  float* part = reinterpret_cast<float*>(smem + p.off_part);
  int* ucnt = reinterpret_cast<int*>(smem + p.off_ucnt);
  uint8_t* xtab = smem + p.off_xtab;
  float* xsx = reinterpret_cast<float*>(smem + p.off_xsx);
  uint8_t* stages = smem + p.off_stage;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = kConsumerWarps;
  constexpr int NC = W * 32;
  const int S = p.nstages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], kProducerThreads);
      mbar_init(&empty[s], W);
    }
    ctl->abort = 0;
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < S; i += blockDim.x) ucnt[i] = 0;
  const int U = p.d / 16;
  const int u0 = (int)((long long)blockIdx.x * U / gridDim.x), u1 = (int)((long long)(blockIdx.x + 1) * U / gridDim.x);
  const int nU = u1 - u0, nseg = p.n / kSegElems;
  // the weight rows do not depend on the previous kernel: start them toward
  // L2 while it finishes
  if (p.prefetch_bytes && threadIdx.x == 0 && nU > 0)
    prefetch_l2(p.W + (size_t)(16 * u0) * p.sg.rb,
                (uint32_t)min((uint64_t)(16 * nU) * p.sg.rb, (uint64_t)p.prefetch_bytes));
  pdl_launch_dependents();
  pdl_wait();
  __syncthreads();

  if (warp >= W) {
    const int ptid = threadIdx.x - NC;
    for (int v = 0; v < nU; v++) {
      const int slot = v % S;
      if (!warp_wait(&empty[slot], (((uint32_t)(v / S)) & 1u) ^ 1u, ctl, p.err)) break;
      const uint8_t* src = p.W + (size_t)(16 * (u0 + v)) * p.sg.rb;
      issue_unit(stages + (size_t)slot * p.stage_bytes, &full[slot], src, src + 8 * (size_t)p.sg.rb, p.sg, ptid,
                 kProducerThreads);
    }
    cp_async_wait_all();
    return;
  }
  // x table (consumers only; the producers already stream weights)
  {
    float* xs = reinterpret_cast<float*>(smem + p.off_stg);
    if (((uintptr_t)p.x & 15) == 0 && (p.n & 3) == 0) {
      stage_vec(p.x, xs, p.n, threadIdx.x, NC, false);
    } else {
      for (int i = threadIdx.x; i < p.n; i += NC) xs[i] = __ldg(p.x + i);
    }
    named_bar(1, NC);
    if (p.norm_w) {
      // x * (1 / sqrt(mean(x^2) + eps)) * w, every CTA on its own copy
      float ss = 0.f;
      for (int i = threadIdx.x; i < p.n; i += NC) ss += xs[i] * xs[i];
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) ctl->nred[warp] = ss;
      named_bar(1, NC);
      float tot = 0.f;
      for (int w = 0; w < W; w++) tot += ctl->nred[w];
      const float r = 1.0f / sqrtf(tot / (float)p.n + p.eps);
      for (int i = threadIdx.x; i < p.n; i += NC) xs[i] = xs[i] * r * __ldg(p.norm_w + i);
      named_bar(1, NC);
    }
    build_tables<SF>(xs, xtab, xsx, p.n / kSegElems, warp, W, lane);
    named_bar(1, NC);
  }
  const LaneCtx L = lane_ctx();
  BFrag bf;
  bf.reset();
  for (int v = 0; v < nU; v++) {
    const int slot = v % S;
    const bool ok = warp_wait(&full[slot], (uint32_t)(v / S) & 1u, ctl, p.err);
    float val = 0.f;
    const bool last = consume<SF>(stages + (size_t)slot * p.stage_bytes, p.sg, v, nseg, warp, xtab, xsx,
                                  part + slot * p.part_stride, &ucnt[slot], L, &val, ok, bf);
    if (last && ok && lane < 16) p.y[16 * (u0 + v) + lane] = val;
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static uint32_t gcd_u(uint32_t a, uint32_t b) {
  while (b) {
    uint32_t t = a % b;
    a = b;
    b = t;
  }
  return a;
}

bool fast_format(uint32_t type) { return type == T_Q8_0 || type == T_Q4_K || type == T_Q6_K; }

int stage_geom(uint32_t type, int K, StageGeom* sg) {
  if (!fast_format(type) || K <= 0 || K % kSegElems) return VIREO_ERR_UNSUPPORTED;
  int be, bb;
  if (type_block(type, &be, &bb)) return VIREO_ERR_UNSUPPORTED;
  const uint32_t rb = (uint32_t)(K / be) * (uint32_t)bb;
  uint32_t G = 16u / gcd_u(rb, 16u);
  if (G > 8) return VIREO_ERR_UNSUPPORTED;
  if ((type == T_Q8_0 || type == T_Q4_K) && G != 1) return VIREO_ERR_UNSUPPORTED;
  const uint32_t gbytes = G * rb;
  const uint32_t pad = (16u - gbytes % 128u + 128u) % 128u;
  sg->rb = rb;
  sg->G = G;
  sg->gstride = gbytes + pad;
  sg->hstride = (8u / G) * sg->gstride;
  // multiply-shift division by gbytes, verified exact over the half's range
  const uint64_t magic = ((1ull << 32) + gbytes - 1) / gbytes;
  if (magic > 0xFFFFFFFFull) return VIREO_ERR_UNSUPPORTED;
  sg->gmagic = (uint32_t)magic;
  for (uint32_t b = 0; b < 8u * rb; b += 16u)
    if ((uint32_t)(((uint64_t)b * sg->gmagic) >> 32) != b / gbytes) return VIREO_ERR_UNSUPPORTED;
  return VIREO_OK;
}

static uint32_t up_to(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

template <class SG, class SD>
static const void* moe_kernel_ptr(bool routed) {
  return routed ? reinterpret_cast<const void*>(&moe_routed_kernel<SG, SD>)
                : reinterpret_cast<const void*>(&moe_decode_kernel<SG, SD>);
}

template <class SG>
static const void* moe_kernel_for(uint32_t dtype, bool routed) {
  if (dtype == T_Q8_0) return moe_kernel_ptr<SG, SegQ8>(routed);
  if (dtype == T_Q4_K) return moe_kernel_ptr<SG, SegQ4K>(routed);
  if (dtype == T_Q6_K) return moe_kernel_ptr<SG, SegQ6K>(routed);
  return nullptr;
}

const void* moe_decode_kernel_for(uint32_t gtype, uint32_t dtype, bool routed) {
  if (gtype == T_Q8_0) return moe_kernel_for<SegQ8>(dtype, routed);
  if (gtype == T_Q4_K) return moe_kernel_for<SegQ4K>(dtype, routed);
  if (gtype == T_Q6_K) return moe_kernel_for<SegQ6K>(dtype, routed);
  return nullptr;
}

// Shared-memory layout for the MoE kernel; picks the deepest stage ring that
// fits.  Returns the dynamic shared-memory bytes (0 if nothing fits).
uint32_t moe_decode_layout(MoeDecodeParams* p, uint32_t smem_limit, int grid) {
  (void)grid;
  const int W = kConsumerWarps;
  const uint32_t stage = up_to(std::max(2u * p->sg_gu.hstride, 2u * p->sg_d.hstride), 128u);
  const uint32_t dslot = up_to(2u * p->sg_d.hstride, 128u);
  p->stage_bytes = stage;
  p->dslot_bytes = dslot;
  p->htab_bytes = (uint32_t)(4 * p->fe);
  const uint32_t htab_region = std::max((uint32_t)p->k * p->htab_bytes, (uint32_t)(4 * p->ne));
  const uint32_t stg_bytes = (uint32_t)std::max(4 * p->d, 4 * p->k);
  p->part_stride = (uint32_t)std::max(W, std::max(p->d, p->fe) / kSegElems) * 16u;
  for (int S = kMaxStages; S >= 2; S--) {
    const int SD = (int)std::min<uint32_t>((uint32_t)kMaxStages, (uint32_t)S * stage / dslot);
    uint32_t off = 4u * kMaxStages * 8u;  // full/empty barriers of both rings
    p->off_ctl = off;
    off = up_to(off + (uint32_t)sizeof(Ctl), 16);
    p->off_part = off;
    off = up_to(off + (uint32_t)S * p->part_stride * 4u, 16);
    p->off_part_d = off;
    off = up_to(off + (uint32_t)SD * p->part_stride * 4u, 16);
    p->off_ucnt = off;
    off = up_to(off + (uint32_t)(2 * kMaxStages * 4), 16);
    p->off_ytile = off;
    off = up_to(off + (uint32_t)(2 * p->k * 16 * 4), 16);
    p->off_xtab = off;
    off = up_to(off + (uint32_t)(4 * p->d), 16);
    p->off_xsx = off;
    off = up_to(off + (uint32_t)(p->d / kSegElems * kMeta * 4), 16);
    p->off_htab = off;
    off = up_to(off + htab_region, 16);
    p->off_hsx = off;
    off = up_to(off + (uint32_t)(p->k * (p->fe / kSegElems) * kMeta * 4), 16);
    p->off_stg = off;
    off = up_to(off + stg_bytes, 128);
    p->off_stage = off;
    off += (uint32_t)S * stage + 16;
    if (off <= smem_limit && SD >= 1) {
      p->nstages = S;
      p->nstages_d = SD;
      return off;
    }
  }
  return 0;
}

const void* gemv_kernel_for(uint32_t type) {
  if (type == T_Q8_0) return reinterpret_cast<const void*>(&gemv_kernel<SegQ8>);
  if (type == T_Q4_K) return reinterpret_cast<const void*>(&gemv_kernel<SegQ4K>);
  if (type == T_Q6_K) return reinterpret_cast<const void*>(&gemv_kernel<SegQ6K>);
  return nullptr;
}

// Shared-memory layout for gemv_kernel: the deepest ring that fits, and no
// deeper than the max_units units a CTA streams (at least 2 stages).
uint32_t gemv_layout(GemvParams* p, uint32_t smem_limit, int max_units) {
  const int W = kConsumerWarps;
  const uint32_t stage = up_to(2u * p->sg.hstride, 128u);
  p->stage_bytes = stage;
  p->part_stride = (uint32_t)std::max(W, p->n / kSegElems) * 16u;
  for (int S = std::max(2, std::min(kMaxStages, max_units)); S >= 2; S--) {
    uint32_t off = 2u * kMaxStages * 8u;
    p->off_ctl = off;
    off = up_to(off + (uint32_t)sizeof(Ctl), 16);
    p->off_part = off;
    off = up_to(off + (uint32_t)S * p->part_stride * 4u, 16);
    p->off_ucnt = off;
    off = up_to(off + (uint32_t)(S * 4), 16);
    p->off_xtab = off;
    off = up_to(off + (uint32_t)(4 * p->n), 16);
    p->off_xsx = off;
    off = up_to(off + (uint32_t)(p->n / kSegElems * kMeta * 4), 16);
    p->off_stg = off;
    off = up_to(off + (uint32_t)(4 * p->n), 128);
    p->off_stage = off;
    off += (uint32_t)S * stage + 16;
    if (off <= smem_limit) {
      p->nstages = S;
      return off;
    }
  }
  return 0;
}

}  // namespace vireo
