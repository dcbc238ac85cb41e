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
  int nvalid;
  int t_lo;
  float xinv;
  int ids[kMaxTopK];
  float wts[kMaxTopK];
  float hinv[kMaxTopK];
};

__device__ const int kNeverAbort = 0;

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
                  const float* sx, float* part, int* ucnt, const LaneCtx& L, float* val, bool active) {
  return consume_unit<S>(stage, sg, v, active ? nseg : 0, kConsumerWarps, w, btab, sx, part, ucnt, L, val);
}

// ---------------------------------------------------------------------------
// MoE decode kernel
// ---------------------------------------------------------------------------
template <class SG, class SD>
__global__ void __launch_bounds__(kDecodeThreads, 1) moe_decode_kernel(const __grid_constant__ MoeDecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kDecodeThreads / 32 + 1];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
  float* part = reinterpret_cast<float*>(smem + p.off_part);
  int* ucnt = reinterpret_cast<int*>(smem + p.off_ucnt);
  uint8_t* xtab = smem + p.off_xtab;
  float* xsx = reinterpret_cast<float*>(smem + p.off_xsx);
  uint8_t* htab = smem + p.off_htab;
  float* hsx = reinterpret_cast<float*>(smem + p.off_hsx);
  uint8_t* stages = smem + p.off_stage;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = kConsumerWarps;
  const int G = gridDim.x, cta = blockIdx.x;
  const int d = p.d, fe = p.fe, ne = p.ne, k = p.k, S = p.nstages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    ctl->abort = 0;
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < S; i += blockDim.x) ucnt[i] = 0;
  __syncthreads();

  // ---- phase R: router partial dot products -------------------------------
  if (warp < W) {
    const int nchunk = d / kRouterChunk;
    const int gw = cta * W + warp, nw = G * W;
    for (int task = gw; task < ne * nchunk; task += nw) {
      const int e = task / nchunk, c = task - e * nchunk;
      const float4* row = reinterpret_cast<const float4*>(p.router + (size_t)e * d + (size_t)c * kRouterChunk);
      const float4* xv = reinterpret_cast<const float4*>(p.hb + (size_t)c * kRouterChunk);
      float4 r[4], xx[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        r[i] = __ldg(row + lane + 32 * i);
        xx[i] = __ldg(xv + lane + 32 * i);
      }
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        s = fmaf(r[i].x, xx[i].x, s);
        s = fmaf(r[i].y, xx[i].y, s);
        s = fmaf(r[i].z, xx[i].z, s);
        s = fmaf(r[i].w, xx[i].w, s);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) p.s.logit_part[(size_t)c * ne + e] = s;
    }
  }

  // ---- x table (every CTA builds its own) ---------------------------------
  {
    float m = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) m = fmaxf(m, fabsf(__ldg(p.hb + i)));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      float mm = 0.f;
      for (int i = 0; i < (int)(blockDim.x / 32); i++) mm = fmaxf(mm, red[i]);
      const float sc = pow2_scale(mm);
      red[kDecodeThreads / 32] = sc;
      ctl->xinv = 1.f / sc;
    }
    __syncthreads();
    build_btab<SG>(p.hb, d, red[kDecodeThreads / 32], xtab, xsx, threadIdx.x, blockDim.x, false);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!grid_barrier(p.s.gsync, (unsigned)G, p.s.err)) ctl->abort = 1;
  }
  __syncthreads();

  // ---- softmax + greedy top-k (every CTA, warp 0) ------------------------
  if (warp == 0 && !aborted(ctl)) {
    const int nchunk = d / kRouterChunk;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int e = lane + 32 * i;
      float s = -INFINITY;
      if (e < ne) {
        s = 0.f;
        for (int c = 0; c < nchunk; c++) s += __ldcg(p.s.logit_part + (size_t)c * ne + e);
      }
      v[i] = s;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; i++) mx = fmaxf(mx, v[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int e = lane + 32 * i;
      v[i] = (e < ne) ? expf(v[i] - mx) : 0.f;
      sum += v[i];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = v[i] / sum;
    uint32_t used = 0;
    for (int t = 0; t < k; t++) {
      float bv = -1.f;
      int bi = -1;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int e = lane + 32 * i;
        if (e < ne && !((used >> i) & 1u) && v[i] > bv) {
          bv = v[i];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi >= 0 && (bi < 0 || oi < bi))) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi >= 0 && (bi & 31) == lane) used |= 1u << (bi >> 5);
      if (lane == 0) {
        ctl->ids[t] = bi;
        ctl->wts[t] = bv;
      }
    }
    __syncwarp();
    if (lane == 0) {
      int nv = 0;
      float ws = 0.f;
      for (int t = 0; t < k; t++) {
        ws = ws + ctl->wts[t];
        nv += ctl->ids[t] >= 0;
      }
      if (p.renorm && ws > 0.f)
        for (int t = 0; t < k; t++) ctl->wts[t] = ctl->wts[t] / ws;
      ctl->nvalid = nv;
      if (cta == 0) {
        for (int t = 0; t < k; t++) {
          if (p.ids_out) p.ids_out[t] = ctl->ids[t];
          if (p.wts_out) p.wts_out[t] = ctl->wts[t];
        }
      }
    }
  }
  __syncthreads();

  // ---- units ---------------------------------------------------------------
  const int rgG = fe / 8, rgD = d / 16;
  const int UG = k * rgG, UD = k * rgD;
  const int g0 = (int)((long long)cta * UG / G), g1 = (int)((long long)(cta + 1) * UG / G);
  const int d0 = (int)((long long)cta * UD / G), d1 = (int)((long long)(cta + 1) * UD / G);
  const int nG = g1 - g0, nD = d1 - d0, nU = nG + nD;
  const int nsegG = d / kSegElems, nsegD = fe / kSegElems;

  if (warp == W) {
    // ---- producer -----------------------------------------------------------
    if (lane == 0) {
      int issued = 0;
      for (int v = 0; v < nU; v++) {
        if (aborted(ctl)) break;
        const int slot = v % S;
        const uint32_t par = ((uint32_t)(v / S) & 1u) ^ 1u;
        if (!mbar_wait(&empty[slot], par, &ctl->abort)) {
          do_abort(ctl, p.s.err, VIREO_ERR_TIMEOUT);
          break;
        }
        uint8_t* stage = stages + (size_t)slot * p.stage_bytes;
        if (v < nG) {
          const int u = g0 + v, t = u / rgG, rg = u - t * rgG;
          const int e = ctl->ids[t];
          if (e < 0) {
            mbar_arrive(&full[slot]);
          } else {
            const uint8_t* gsrc = p.exp_tab[3 * e + 0] + (size_t)(8 * rg) * p.sg_gu.rb;
            const uint8_t* usrc = p.exp_tab[3 * e + 1] + (size_t)(8 * rg) * p.sg_gu.rb;
            issue_unit(stage, &full[slot], gsrc, usrc, p.sg_gu);
          }
        } else {
          const int u = d0 + (v - nG), t = u / rgD, rg = u - t * rgD;
          const int e = ctl->ids[t];
          if (e < 0) {
            mbar_arrive(&full[slot]);
          } else {
            const uint8_t* src = p.exp_tab[3 * e + 2] + (size_t)(16 * rg) * p.sg_d.rb;
            issue_unit(stage, &full[slot], src, src + 8 * (size_t)p.sg_d.rb, p.sg_d);
          }
        }
        issued = v + 1;
      }
      // drain: every copy this CTA issued must land before the CTA exits
      for (int v = (issued > S ? issued - S : 0); v < issued; v++)
        mbar_wait(&full[v % S], (uint32_t)(v / S) & 1u, &kNeverAbort);
    }
    return;
  }

  // ---- consumers -------------------------------------------------------------
  const LaneCtx L = lane_ctx();
  for (int v = 0; v < nG; v++) {
    const int slot = v % S;
    bool ok = !aborted(ctl) && mbar_wait(&full[slot], (uint32_t)(v / S) & 1u, &ctl->abort);
    if (!ok && !aborted(ctl)) do_abort(ctl, p.s.err, VIREO_ERR_TIMEOUT);
    const int u = g0 + v, t = u / rgG, rg = u - t * rgG;
    const bool active = ok && ctl->ids[t] >= 0;
    float val = 0.f;
    const bool last = consume<SG>(stages + (size_t)slot * p.stage_bytes, p.sg_gu, v, nsegG, warp, xtab, xsx,
                                  part + slot * W * 16, &ucnt[slot], L, &val, active);
    if (last) {
      const float up = __shfl_sync(0xffffffffu, val, (lane + 8) & 31);
      if (active && lane < 8) {
        const float gg = val * ctl->xinv, uu = up * ctl->xinv;
        const float sl = gg / (1.0f + expf(-gg));
        p.s.hbuf[(size_t)t * fe + 8 * rg + lane] = sl * uu;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  // ---- phase boundary: every h row of every expert is written --------------
  named_bar(1, W * 32);
  if (threadIdx.x == 0 && !aborted(ctl)) {
    if (!grid_barrier(p.s.gsync, (unsigned)G, p.s.err)) ctl->abort = 1;
  }
  named_bar(1, W * 32);
  const int t_lo = (nD > 0) ? d0 / rgD : 0;
  const int t_hi = (nD > 0) ? (d1 - 1) / rgD : -1;
  if (!aborted(ctl)) {
    for (int t = t_lo + warp; t <= t_hi; t += W) {
      if (ctl->ids[t] < 0) continue;
      const float* hv = p.s.hbuf + (size_t)t * fe;
      float m = 0.f;
      for (int i = lane; i < fe; i += 32) m = fmaxf(m, fabsf(__ldcg(hv + i)));
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float sc = pow2_scale(m);
      if (lane == 0) ctl->hinv[t] = 1.f / sc;
      build_btab<SD>(hv, fe, sc, htab + (size_t)(t - t_lo) * p.htab_bytes, hsx + (size_t)(t - t_lo) * (fe / 32),
                     lane, 32, true);
    }
  }
  named_bar(1, W * 32);

  for (int v = nG; v < nU; v++) {
    const int slot = v % S;
    bool ok = !aborted(ctl) && mbar_wait(&full[slot], (uint32_t)(v / S) & 1u, &ctl->abort);
    if (!ok && !aborted(ctl)) do_abort(ctl, p.s.err, VIREO_ERR_TIMEOUT);
    const int u = d0 + (v - nG), t = u / rgD, rg = u - t * rgD;
    const bool active = ok && ctl->ids[t] >= 0;
    float val = 0.f;
    const bool last = consume<SD>(stages + (size_t)slot * p.stage_bytes, p.sg_d, v, nsegD, warp,
                                  htab + (size_t)(t - t_lo) * p.htab_bytes, hsx + (size_t)(t - t_lo) * (fe / 32),
                                  part + slot * W * 16, &ucnt[slot], L, &val, active);
    if (last && active) {
      if (lane < 16) p.s.ybuf[(size_t)t * d + 16 * rg + lane] = val * ctl->hinv[t];
      __syncwarp();
      unsigned int old = 0;
      if (lane == 0) {
        __threadfence();
        old = atomicAdd(&p.s.tile_cnt[rg], 1u);
        __threadfence();
      }
      old = __shfl_sync(0xffffffffu, old, 0);
      if ((int)old == ctl->nvalid - 1) {
        __syncwarp();
        if (lane < 16) {
          const int r = 16 * rg + lane;
          float acc = 0.f;
          for (int tt = 0; tt < k; tt++)
            if (ctl->ids[tt] >= 0) acc = __fadd_rn(acc, __fmul_rn(ctl->wts[tt], __ldcg(p.s.ybuf + (size_t)tt * d + r)));
          p.x[r] = __fadd_rn(p.x[r], acc);
        }
        if (lane == 0) atomicExch(&p.s.tile_cnt[rg], 0u);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
}

// ---------------------------------------------------------------------------
// Stand-alone GEMV: y[d] = W[d x n] . x[n]  (fast formats, d % 16 == 0)
// ---------------------------------------------------------------------------
template <class SF>
__global__ void __launch_bounds__(kDecodeThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kDecodeThreads / 32 + 1];
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
  const int S = p.nstages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    ctl->abort = 0;
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < S; i += blockDim.x) ucnt[i] = 0;
  const int U = p.d / 16;
  const int u0 = (int)((long long)blockIdx.x * U / gridDim.x), u1 = (int)((long long)(blockIdx.x + 1) * U / gridDim.x);
  const int nU = u1 - u0, nseg = p.n / kSegElems;
  __syncthreads();

  if (warp == W) {
    if (lane == 0) {
      int issued = 0;
      for (int v = 0; v < nU; v++) {
        if (aborted(ctl)) break;
        const int slot = v % S;
        if (!mbar_wait(&empty[slot], (((uint32_t)(v / S)) & 1u) ^ 1u, &ctl->abort)) {
          do_abort(ctl, p.err, VIREO_ERR_TIMEOUT);
          break;
        }
        const uint8_t* src = p.W + (size_t)(16 * (u0 + v)) * p.sg.rb;
        issue_unit(stages + (size_t)slot * p.stage_bytes, &full[slot], src, src + 8 * (size_t)p.sg.rb, p.sg);
        issued = v + 1;
      }
      for (int v = (issued > S ? issued - S : 0); v < issued; v++)
        mbar_wait(&full[v % S], (uint32_t)(v / S) & 1u, &kNeverAbort);
    }
    return;
  }
  // x table (consumers only; the producer already streams weights)
  {
    float m = 0.f;
    for (int i = threadIdx.x; i < p.n; i += W * 32) m = fmaxf(m, fabsf(__ldg(p.x + i)));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    named_bar(1, W * 32);
    if (threadIdx.x == 0) {
      float mm = 0.f;
      for (int i = 0; i < W; i++) mm = fmaxf(mm, red[i]);
      const float sc = pow2_scale(mm);
      red[W] = sc;
      ctl->xinv = 1.f / sc;
    }
    named_bar(1, W * 32);
    build_btab<SF>(p.x, p.n, red[W], xtab, xsx, threadIdx.x, W * 32, false);
    named_bar(1, W * 32);
  }
  const LaneCtx L = lane_ctx();
  for (int v = 0; v < nU; v++) {
    const int slot = v % S;
    bool ok = !aborted(ctl) && mbar_wait(&full[slot], (uint32_t)(v / S) & 1u, &ctl->abort);
    if (!ok && !aborted(ctl)) do_abort(ctl, p.err, VIREO_ERR_TIMEOUT);
    float val = 0.f;
    const bool last = consume<SF>(stages + (size_t)slot * p.stage_bytes, p.sg, v, nseg, warp, xtab, xsx,
                                  part + slot * W * 16, &ucnt[slot], L, &val, ok);
    if (last && ok && lane < 16) p.y[16 * (u0 + v) + lane] = val * ctl->xinv;
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
  return VIREO_OK;
}

static uint32_t up_to(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

template <class SG, class SD>
static const void* moe_kernel_ptr() {
  return reinterpret_cast<const void*>(&moe_decode_kernel<SG, SD>);
}

template <class SG>
static const void* moe_kernel_for(uint32_t dtype) {
  if (dtype == T_Q8_0) return moe_kernel_ptr<SG, SegQ8>();
  if (dtype == T_Q4_K) return moe_kernel_ptr<SG, SegQ4K>();
  if (dtype == T_Q6_K) return moe_kernel_ptr<SG, SegQ6K>();
  return nullptr;
}

const void* moe_decode_kernel_for(uint32_t gtype, uint32_t dtype) {
  if (gtype == T_Q8_0) return moe_kernel_for<SegQ8>(dtype);
  if (gtype == T_Q4_K) return moe_kernel_for<SegQ4K>(dtype);
  if (gtype == T_Q6_K) return moe_kernel_for<SegQ6K>(dtype);
  return nullptr;
}

// Shared-memory layout for the MoE kernel; picks the deepest stage ring that
// fits.  Returns the dynamic shared-memory bytes (0 if nothing fits).
uint32_t moe_decode_layout(MoeDecodeParams* p, uint32_t smem_limit) {
  const int W = kConsumerWarps;
  const uint32_t stage = up_to(std::max(2u * p->sg_gu.hstride, 2u * p->sg_d.hstride), 128u);
  p->stage_bytes = stage;
  p->htab_bytes = (uint32_t)(4 * p->fe);
  for (int S = kMaxStages; S >= 2; S--) {
    uint32_t off = 2u * kMaxStages * 8u;
    p->off_ctl = off;
    off = up_to(off + (uint32_t)sizeof(Ctl), 16);
    p->off_part = off;
    off = up_to(off + (uint32_t)(S * W * 16 * 4), 16);
    p->off_ucnt = off;
    off = up_to(off + (uint32_t)(S * 4), 16);
    p->off_xtab = off;
    off = up_to(off + (uint32_t)(4 * p->d), 16);
    p->off_xsx = off;
    off = up_to(off + (uint32_t)(p->d / 32 * 4), 16);
    p->off_htab = off;
    off = up_to(off + (uint32_t)p->k * p->htab_bytes, 16);
    p->off_hsx = off;
    off = up_to(off + (uint32_t)(p->k * (p->fe / 32) * 4), 128);
    p->off_stage = off;
    off += (uint32_t)S * stage + 16;
    if (off <= smem_limit) {
      p->nstages = S;
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

uint32_t gemv_layout(GemvParams* p, uint32_t smem_limit) {
  const int W = kConsumerWarps;
  const uint32_t stage = up_to(2u * p->sg.hstride, 128u);
  p->stage_bytes = stage;
  for (int S = kMaxStages; S >= 2; S--) {
    uint32_t off = 2u * kMaxStages * 8u;
    p->off_ctl = off;
    off = up_to(off + (uint32_t)sizeof(Ctl), 16);
    p->off_part = off;
    off = up_to(off + (uint32_t)(S * W * 16 * 4), 16);
    p->off_ucnt = off;
    off = up_to(off + (uint32_t)(S * 4), 16);
    p->off_xtab = off;
    off = up_to(off + (uint32_t)(4 * p->n), 16);
    p->off_xsx = off;
    off = up_to(off + (uint32_t)(p->n / 32 * 4), 128);
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
