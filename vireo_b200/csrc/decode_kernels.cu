// Decode kernels: the MoE FFN block (one token per launch, all phases in
// one kernel) and the stand-alone quantised GEMV behind gguf_matmul.  See
// moe_decode.cuh and engine.cuh for the design.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <type_traits>

#include "moe_decode.cuh"
#include "vireo_internal.h"

namespace vireo {

constexpr int kTrItems = 16;  // items with per-item trace stamps

struct Ctl {
  int abort;
  float wsum;  // renorm denominator
  int ids[kMaxTopK];
  float wts[kMaxTopK];
  float nred[kConsumerWarps];  // gemv_kernel: per-warp sums of squares for the fused norm
  float sred[kConsumerWarps + kProducerWarps];  // moe_decode: per-warp sums of squares for the fused norm
  // the item each ring slot holds now (-1: none yet), written by the producer
  // before it issues the item's copies
  int slot_item[kMaxStages];
  // trace only: first full-wait return and last empty arrival of the first items
  unsigned long long it_land[kTrItems], it_done[kTrItems];
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

// Warp-collective wait for item i's data in its ring slot.  A warp that owns
// only some items may reach item i while the slot still holds item i - S, in
// which case a parity wait alone would see the earlier phase and return at
// once; so the warp first waits (bounded) until the producer has recorded
// item i in the slot, and only then waits on the full barrier's parity.
VDEV bool item_wait(uint64_t* full, Ctl* ctl, int* err, int i, int S) {
  const int slot = i % S;
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    const volatile int* rec = &ctl->slot_item[slot];
    if (*rec != i) {
      const uint64_t t0 = now_ns();
      while (*rec != i) {
        if (aborted(ctl)) {
          ok = 0;
          break;
        }
        if (now_ns() - t0 > kWaitLimitNs) {
          do_abort(ctl, err, VIREO_ERR_TIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(32);
      }
    }
    if (ok) ok = (!aborted(ctl) && mbar_wait(&full[slot], (uint32_t)(i / S) & 1u, &ctl->abort)) ? 1 : 0;
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

// Routing after every CTA's logits are in, in two steps.
//
// route_keys (one warp): the softmax of the ne logits with expf (max
// subtracted; the sum over a lane's experts l, l + 32, ... in order, then
// across lanes by an xor tree) and, per expert, a 64-bit selection key:
// the probability's bits above (p >= 0, so bit order is value order) and
// 0xffffffff - e below, or 0 for NaN.  Key order is the order (p desc, id
// asc) in which the reference's greedy strict-'>' scan from id 0 takes the
// experts (gguf_run.c:190-191), and a NaN key never outranks a valid one.
// Keys past ne up to np (a power of two) are 0.  Slots from the number of
// valid experts to k get id -1 and weight -1, as the reference's scan
// leaves them.
VDEV void route_keys(const MoeDecodeParams& p, Ctl* ctl, unsigned long long* key, int np, int lane) {
  constexpr int kPer = kMaxExperts / 32;
  const int ne = p.ne, k = p.k, R = (ne + 31) / 32;
  float lv[kPer];
#pragma unroll
  for (int i = 0; i < kPer; i++) {
    const int e = lane + 32 * i;
    lv[i] = -INFINITY;
    if (i < R && e < ne) lv[i] = __ldcg(p.s.logit_part + e);
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kPer; i++) m = fmaxf(m, lv[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float ex[kPer], sm = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; i++) {
    ex[i] = (i < R && lane + 32 * i < ne) ? expf(lv[i] - m) : 0.f;
    sm += ex[i];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
  int nvalid = 0;
#pragma unroll
  for (int i = 0; i < kPer; i++) {
    const int e = lane + 32 * i;
    unsigned long long kv = 0ull;
    if (i < R && e < ne) {
      const float pe = ex[i] / sm;
      if (!isnan(pe)) kv = ((unsigned long long)__float_as_uint(pe) << 32) | (0xffffffffu - (unsigned)e);
    }
    nvalid += __popc(__ballot_sync(0xffffffffu, kv != 0ull));
    if (e < np) key[e] = kv;
  }
  for (int t = nvalid + lane; t < k; t += 32) {
    ctl->ids[t] = -1;
    ctl->wts[t] = -1.f;
  }
}

// route_select (every thread of the CTA): expert e's rank is the number of
// keys above its own; Q = threads / np threads share an expert, thread q
// counting the 16-byte key pairs q, q + Q, q + 2Q, ... (the Q threads of an
// expert read Q adjacent pairs: no bank conflicts), summed across the Q
// lanes.  Ranks below k are the selection, in rank order, with the
// probabilities as the weights (renormalisation comes after: route_finish).
VDEV void route_select(Ctl* ctl, const unsigned long long* key, int np, int k) {
  const int nthr = blockDim.x, Q = nthr / np;  // np <= 256 <= nthr / 2: Q >= 2, a power of two
  const int e = threadIdx.x / Q, q = threadIdx.x - e * Q, npair = np / 2 / Q;
  const unsigned long long ke = key[e];
  const ulonglong2* k2 = reinterpret_cast<const ulonglong2*>(key) + q;
  int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
#pragma unroll 4
  for (int j = 0; j < npair; j += 2) {  // npair is even (np >= 64)
    const ulonglong2 v = k2[j * Q], w = k2[(j + 1) * Q];
    r0 += v.x > ke;
    r1 += v.y > ke;
    r2 += w.x > ke;
    r3 += w.y > ke;
  }
  int rank = (r0 + r1) + (r2 + r3);
  for (int o = Q >> 1; o; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
  if (q == 0 && ke != 0ull && rank < k) {
    ctl->ids[rank] = e;
    ctl->wts[rank] = __uint_as_float((unsigned)(ke >> 32));
  }
}

// One warp, after the selection is published: the optional renormalisation
// by the sequential rank-order sum of the weights (gguf_run.c:192), -1 slots
// included as the reference adds them, and the selection out.
VDEV void route_finish(const MoeDecodeParams& p, Ctl* ctl, int lane, bool write_out) {
  const int k = p.k;
  float ws = 0.f;
#pragma unroll 1
  for (int j0 = 0; j0 < k; j0 += 8) {
    float w8[8];  // eight loads in flight, then the adds in order
#pragma unroll
    for (int u = 0; u < 8; u++) w8[u] = j0 + u < k ? ctl->wts[j0 + u] : 0.f;
#pragma unroll
    for (int u = 0; u < 8; u++)
      if (j0 + u < k) ws = ws + w8[u];
  }
  __syncwarp();
  for (int t = lane; t < k; t += 32) {
    float w = ctl->wts[t];
    if (p.renorm && ws > 0.f) w = w / ws;
    ctl->wts[t] = w;
    if (write_out) {
      if (p.ids_out) p.ids_out[t] = ctl->ids[t];
      if (p.wts_out) p.wts_out[t] = w;
    }
  }
  __syncwarp();
}

// Bounded wait on a phase with no early exit on abort: used where bulk
// copies may still be writing this CTA's shared memory (they complete
// whatever the kernel's state), so that the CTA never exits before them.
VDEV bool wait_copies(uint64_t* bar, uint32_t par) {
  const int never = 0;
  return mbar_wait(bar, par, &never);
}

// The producer warp's item loop over one ring: item i goes to slot i % S
// once its previous occupant (item i - S) has been released by every
// consumer warp (empty) and its copies have landed (full), so no two copies
// ever target one slot at once; at the end it waits for the copies of the
// last S items.  issue(i, slot_base) announces the item's bytes on full[slot]
// and issues its copies (warp-collective).  Returns the items issued.
template <class Issue>
VDEV int produce_ring(uint64_t* full, uint64_t* empty, uint8_t* stages, uint32_t stage_bytes, int S, int n,
                      Ctl* ctl, int* err, Issue&& issue) {
  int i = 0;
  for (; i < n; i++) {
    const int slot = i % S;
    if (i >= S) {
      if (!warp_wait(&empty[slot], ((uint32_t)(i / S) & 1u) ^ 1u, ctl, err)) break;
      if ((threadIdx.x & 31) == 0) wait_copies(&full[slot], (uint32_t)((i - S) / S) & 1u);
      __syncwarp();
    }
    if (aborted(ctl)) break;
    // the slot's previous item is released and its copies landed: the full
    // barrier's open phase is item i's from here on
    if ((threadIdx.x & 31) == 0) *reinterpret_cast<volatile int*>(&ctl->slot_item[slot]) = i;
    issue(i, slot, stages + (size_t)slot * stage_bytes);
  }
  if ((threadIdx.x & 31) == 0)
    for (int j = i > S ? i - S : 0; j < i; j++) wait_copies(&full[j % S], (uint32_t)(j / S) & 1u);
  __syncwarp();
  return i;
}

// The decode kernel body.  ROUTED: the route comes from the caller (rt) and
// the router phase is skipped; otherwise every CTA computes it.
template <class SG, class SD, bool ROUTED>
__device__ __forceinline__ void moe_decode_body(const MoeDecodeParams& p, const MoeRoute* rt) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + p.off_ctl);
  const uint8_t** etab = reinterpret_cast<const uint8_t**>(smem + p.off_etab);  // [ne][3] expert slices
  int* ucnt = reinterpret_cast<int*>(smem + p.off_ucnt);  // [S][kMaxDTiles]: [0] = tiles of the item done
  const VecTab xt = {smem + p.off_xtab, reinterpret_cast<float*>(smem + p.off_xmeta), smem + p.off_xrtab,
                     reinterpret_cast<float*>(smem + p.off_xrmeta)};
  const VecTab ht = {smem + p.off_htab, reinterpret_cast<float*>(smem + p.off_hmeta), smem + p.off_hrtab,
                     reinterpret_cast<float*>(smem + p.off_hrmeta)};
  float* xs = reinterpret_cast<float*>(smem + p.off_xs);  // residual rows of this CTA's down tiles
  uint8_t* stages = smem + p.off_stage;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = kConsumerWarps;
  constexpr int NC = W * 32;  // consumer threads
  const int G = gridDim.x, cta = blockIdx.x;
  const int d = p.d, fe = p.fe, ne = p.ne, k = p.k, S = p.nstages;
  MoeSync* sy = p.s.sync;
  // This CTA's share of the work (known before the route, and worked out
  // here, off the serial path): group t (the expert of rank t) = CTAs
  // [t G / k, (t + 1) G / k), i.e. t = ((cta + 1) k - 1) / G; CTA j of the m
  // in the group takes an even share of the expert's fe / 8 gate/up units
  // and of its d / 16 down tiles.
  const int t = ((cta + 1) * k - 1) / G;
  const int c0 = t * G / k, c1 = (t + 1) * G / k;
  const int m = c1 - c0, j = cta - c0;
  const int U = fe / 8, NT = d / 16, P = p.dtiles;
  const int u0 = j * U / m, u1 = (j + 1) * U / m;
  const int i0 = j * NT / m, i1 = (j + 1) * NT / m;

  if (threadIdx.x == 0) {
    trace(p, kTrStart);
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);   // the producer's arrive.expect_tx; the copies complete the bytes
      mbar_init(&empty[s], 1);  // the warp that finishes the item's last unit or tile
      ctl->slot_item[s] = -1;
    }
    ctl->abort = 0;
    mbar_fence_init();
  }
  for (int i = threadIdx.x; i < S * kMaxDTiles; i += blockDim.x) ucnt[i] = 0;
  if (p.trace)
    for (int i = threadIdx.x; i < kTrItems; i += blockDim.x) {
      ctl->it_land[i] = ~0ull;
      ctl->it_done[i] = 0ull;
    }
  // expert slice table (weights metadata: not written by the previous kernel)
  if constexpr (!ROUTED)
    for (int i = threadIdx.x; i < 3 * ne; i += blockDim.x) etab[i] = p.exp_tab[i];
  // the next token's kernel may start its own prologue as SMs free up
  pdl_launch_dependents();

  if constexpr (ROUTED) {
    // ---- caller's route: x tables and the selection, no router phase --------
    pdl_wait();
    stage_vec(p.hb, reinterpret_cast<float*>(xt.tab), d, threadIdx.x, blockDim.x, false);
    if (threadIdx.x < k) {
      ctl->ids[threadIdx.x] = rt->ids[threadIdx.x];
      ctl->wts[threadIdx.x] = rt->wts[threadIdx.x];
      if (cta == 0) {
        if (p.ids_out) p.ids_out[threadIdx.x] = rt->ids[threadIdx.x];
        if (p.wts_out) p.wts_out[threadIdx.x] = rt->wts[threadIdx.x];
      }
    }
    __syncthreads();
    if (p.sh_gate) {
      // a shared expert's gate: sigmoid(g . hb), the dot in every CTA
      const float* xv = reinterpret_cast<const float*>(xt.tab);
      float z = 0.f;
      for (int i = threadIdx.x; i < d; i += blockDim.x) z = fmaf(__ldg(p.sh_gate + i), xv[i], z);
#pragma unroll
      for (int o = 16; o; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
      if (lane == 0) ctl->sred[warp] = z;
      __syncthreads();
      if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int w = 0; w < kConsumerWarps + kProducerWarps; w++) tot += ctl->sred[w];
        ctl->wts[0] = 1.0f / (1.0f + expf(-tot));
      }
      __syncthreads();
    }
    build_tables<SG>(reinterpret_cast<const float*>(xt.tab), xt, d / kSegElems, warp, (int)(blockDim.x / 32), lane);
    __syncthreads();
    if (threadIdx.x == 0) trace(p, kTrRouted);
  } else {
    // ---- phase R: router logits, one warp per expert ----------------------------
    // A warp takes expert e's whole row against x (staged once in shared
    // memory): each lane's products over the row in order, then an xor tree
    // across the warp; the logit goes to scratch.  The row's first four
    // 512-value chunks are weights (independent of the previous kernel):
    // their loads are issued before waiting on the previous kernel.
    const int nchunk = d / kRouterChunk;
    const int nw = G * (int)(blockDim.x / 32);
    const int gw = warp * G + cta;  // spread experts over all CTAs first
    constexpr int kPre = 4;         // chunks held in registers across the wait
    float4 rp[kPre][4];
    if (gw < ne) {
#pragma unroll
      for (int c = 0; c < kPre; c++)
        if (c < nchunk) {
          const float4* row = reinterpret_cast<const float4*>(p.router + (size_t)gw * d + (size_t)c * kRouterChunk);
#pragma unroll
          for (int i = 0; i < 4; i++) rp[c][i] = __ldg(row + lane + 32 * i);
        }
    }
    pdl_wait();
    if (threadIdx.x == 0) trace(p, kTrPdl);
    const float* xsm = reinterpret_cast<const float*>(xt.tab);
    if (p.norm_w) {
      // the decoder's x += attention output, xb = ffn_norm(x) (gguf_run.c:
      // 237-238, rmsnorm :161-165), formed by every CTA into the staged vector
      float* xv = reinterpret_cast<float*>(xt.tab);
      float ss = 0.f;
      for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = p.x[i] + p.res_y[i];
        xv[i] = v;
        ss += v * v;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) ctl->sred[warp] = ss;
      __syncthreads();
      ss = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps + kProducerWarps; w++) ss += ctl->sred[w];
      const float r = 1.0f / sqrtf(ss / (float)d + p.norm_eps);
      for (int i = threadIdx.x; i < d; i += blockDim.x) xv[i] = xv[i] * r * p.norm_w[i];
    } else {
      stage_vec(p.hb, reinterpret_cast<float*>(xt.tab), d, threadIdx.x, blockDim.x, false);
    }
    __syncthreads();
    for (int e = gw; e < ne; e += nw) {
      float v = 0.f;
#pragma unroll 1
      for (int c = 0; c < nchunk; c++) {
        float4 r[4];
        if (e == gw && c < kPre) {
#pragma unroll
          for (int cc = 0; cc < kPre; cc++)
            if (cc == c) {
#pragma unroll
              for (int i = 0; i < 4; i++) r[i] = rp[cc][i];
            }
        } else {
          const float4* row = reinterpret_cast<const float4*>(p.router + (size_t)e * d + (size_t)c * kRouterChunk);
#pragma unroll
          for (int i = 0; i < 4; i++) r[i] = __ldg(row + lane + 32 * i);
        }
        const float4* xv = reinterpret_cast<const float4*>(xsm + (size_t)c * kRouterChunk);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float4 xx = xv[lane + 32 * i];
          v = fmaf(r[i].x, xx.x, v);
          v = fmaf(r[i].y, xx.y, v);
          v = fmaf(r[i].z, xx.z, v);
          v = fmaf(r[i].w, xx.w, v);
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) p.s.logit_part[e] = v;
    }
    __syncthreads();  // this CTA's logits are written
    if (warp == W && lane == 0) {
      trace(p, kTrRouterDone);
      red_add_release_gpu(&sy->router_arrive.v, 1u);
      if (!wait_geq(&sy->router_arrive.v, (unsigned)G, p.s.err)) ctl->abort = 1;
      trace(p, kTrPartials);
    }
    __syncthreads();  // every CTA's logits are in (or the wait gave up)
    // selection keys in the h table area (idle until the down phase)
    int np = 64;
    while (np < ne) np <<= 1;
    unsigned long long* key = reinterpret_cast<unsigned long long*>(ht.tab);
    const bool go = !aborted(ctl);
    if (go && warp == 0) route_keys(p, ctl, key, np, lane);
    __syncthreads();
    if (go) route_select(ctl, key, np, k);
    __syncthreads();  // the selection (weights not yet renormalised)
    if (warp == W) {
      if (lane == 0) trace(p, kTrRouted);
    } else {
      // consumer warp 0 renormalises the weights and writes the selection
      // out while the others build the x tables (in place over the staged
      // x); the producer starts on the copies at once
      if (warp == 0 && go) route_finish(p, ctl, lane, cta == 0);
      build_tables<SG>(xsm, xt, d / kSegElems, warp, W, lane);
      named_bar(1, NC);
    }
  }

  // ---- this CTA's share of the selected expert of rank t ----------------------
  const bool active = !aborted(ctl) && ctl->ids[t] >= 0;
  const int nG = active ? u1 - u0 : 0, nD = i1 - i0;  // an unused slot still counts its tiles
  const int nDI = active ? (nD + P - 1) / P : 0;    // down items (up to P tiles per stage)
  const int nItems = nG + nDI;
  const uint8_t* gsl = nullptr;
  const uint8_t* usl = nullptr;
  const uint8_t* dsl = nullptr;
  if (active) {
    if constexpr (ROUTED) {
      gsl = rt->ptr[t][0];
      usl = rt->ptr[t][1];
      dsl = rt->ptr[t][2];
    } else {
      const int e = ctl->ids[t];
      gsl = etab[3 * e + 0];
      usl = etab[3 * e + 1];
      dsl = etab[3 * e + 2];
    }
  }

  if (warp >= W) {
    // ---- producer warp: bulk copies of the items, in ring order ---------------
    if (lane == 0) trace(p, kTrProdFirst);
    if (active) {
      produce_ring(full, empty, stages, p.stage_bytes, S, nItems, ctl, p.s.err, [&](int i, int slot, uint8_t* st) {
        if (p.trace && lane == 0 && i < kTrItems) p.trace[blockIdx.x * kTraceSlots + 16 + i] = now_ns();
        if (i < nG) {
          if (lane == 0) mbar_arrive_expect_tx(&full[slot], 16u * p.sg_gu.rb);
          __syncwarp();
          const size_t row = (size_t)(8 * (u0 + i)) * p.sg_gu.rb;
          issue_tile_bulk(st, &full[slot], gsl + row, usl + row, p.sg_gu, lane);
        } else {
          if (i == nG && lane == 0) trace(p, kTrProdFirstD);
          const int tt0 = (i - nG) * P, nt = min(P, nD - tt0);
          if (lane == 0) mbar_arrive_expect_tx(&full[slot], (uint32_t)nt * 16u * p.sg_d.rb);
          __syncwarp();
          for (int tt = 0; tt < nt; tt++) {
            const uint8_t* src = dsl + (size_t)(16 * (i0 + tt0 + tt)) * p.sg_d.rb;
            issue_tile_bulk(st + (size_t)tt * p.dslot_bytes, &full[slot], src, src + 8 * (size_t)p.sg_d.rb, p.sg_d,
                            lane);
          }
        }
      });
    }
    if (lane == 0) trace(p, kTrProdDrained);
    return;
  }

  // ---- consumers ----------------------------------------------------------------
  for (int i = threadIdx.x; i < 16 * nD; i += NC)
    xs[i] = p.norm_w ? p.x[16 * i0 + i] + p.res_y[16 * i0 + i] : p.x[16 * i0 + i];
  const LaneCtx L = lane_ctx();
  const int nsg = d / kSegElems, nsd = fe / kSegElems;
  BFrag bf;
  bf.reset();

  // count one finished down tile; the last of the k experts to finish it
  // combines them in the reference's order (acc = sum over rank tt of
  // w_tt * y_tt, then x += acc) into the residual
  auto count_tile = [&](int tile) {  // after the down rows were fenced (below)
    int last = 0;
    if (lane == 0) last = atomicAdd(&p.s.tile_cnt[(size_t)tile * kTileCntStride], 1u) == (unsigned)(k - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      if (lane < 16 && !aborted(ctl)) {
        const int row = 16 * tile + lane;
        float acc = 0.f;
#pragma unroll 1
        for (int t0 = 0; t0 < k; t0 += 8) {
          float yv[8];  // eight experts' rows in flight at once
#pragma unroll
          for (int u = 0; u < 8; u++)
            yv[u] = (t0 + u < k && ctl->ids[t0 + u] >= 0) ? __ldcg(p.s.ybuf + (size_t)(t0 + u) * d + row) : 0.f;
#pragma unroll
          for (int u = 0; u < 8; u++)
            if (t0 + u < k && ctl->ids[t0 + u] >= 0) acc = __fadd_rn(acc, __fmul_rn(ctl->wts[t0 + u], yv[u]));
        }
        p.x[row] = __fadd_rn(xs[16 * (tile - i0) + lane], acc);
      }
      __syncwarp();
      if (lane == 0) p.s.tile_cnt[(size_t)tile * kTileCntStride] = 0u;
    }
  };

  // the G -> D boundary: publish this CTA's units, wait for the group's, then
  // stage the expert's h and build its tables
  auto g_to_d = [&](bool need_h) {
    __threadfence();  // this warp's h values before the group's count
    named_bar(1, NC);
    if (threadIdx.x == 0) {
      trace(p, kTrGDone);
      if (nG > 0) red_add_release_gpu(&sy->group[t].v, (unsigned)nG);
      if (need_h && !aborted(ctl) && !wait_geq(&sy->group[t].v, (unsigned)U, p.s.err)) ctl->abort = 1;
      trace(p, kTrGAll);
    }
    if (!need_h) return;
    // every warp meets the same barriers whatever the abort flag says (the
    // producer may set it at any time): it only decides whether work is done
    named_bar(1, NC);
    if (!aborted(ctl))
      stage_vec_cg8(p.s.hbuf + (size_t)t * fe, reinterpret_cast<float*>(ht.tab), fe, threadIdx.x, NC);
    named_bar(1, NC);
    if (!aborted(ctl)) build_tables<SD>(reinterpret_cast<const float*>(ht.tab), ht, nsd, warp, W, lane);
    named_bar(1, NC);
    if (threadIdx.x == 0) trace(p, kTrHtab);
  };

  // Units and tiles go to warp groups; with pairs, warp 2q + hf of pair q
  // runs half hf of the segments (the first half the lower ones), the pair adds the two
  // halves' row sums in that order through shared memory (a double buffer
  // by iteration parity, so a warp one iteration ahead never overwrites
  // sums its partner has not read), and warp 2q finishes the row values.
  // Warps per unit or tile: two for Q8_0 gate/up rows (the heaviest
  // segment kernel: a pair halves the per-unit latency that bounds the ring's
  // turnover), one for the lighter formats, where the pair's exchange cost
  // more than it saved (measured on the OLMoE- and Qwen3-shaped layers).
  constexpr int WPU = std::is_same<SG, SegQ8>::value ? 2 : 1;
  constexpr int NP = W / WPU;  // warp groups; with pairs, a last odd warp idles in these phases
  const int q = warp / WPU, hf = warp % WPU;
  float* pbuf = reinterpret_cast<float*>(smem + p.off_part) + (WPU == 2 ? q * 32 : 0);  // [2 parities][16]
  auto pair_sum = [&](float& v0, float& v1, int iter) {
    if constexpr (WPU == 1) return;
    float* pb = pbuf + 16 * (iter & 1);
    if (hf && L.t == 0) {
      pb[L.g] = v0;
      pb[8 + L.g] = v1;
    }
    named_bar(4 + q, 64);
    if (!hf && L.t == 0) {
      v0 += pb[L.g];
      v1 += pb[8 + L.g];
    }
  };

  // ---- gate/up units: unit i to pair i mod NP ----------------------------------
  const int nsg_lo = WPU == 2 ? nsg / 2 : nsg, nsd_lo = WPU == 2 ? nsd / 2 : nsd;
  if (q < NP) {
#pragma unroll 1
    for (int i = q, it = 0; i < nG; i += NP, it++) {
      const int slot = i % S;
      const bool ok = item_wait(full, ctl, p.s.err, i, S);
      if (p.trace && lane == 0 && !hf && i < kTrItems) atomicMin(&ctl->it_land[i], now_ns());
      const uint8_t* st = stages + (size_t)slot * p.stage_bytes;
      const uint8_t* r0 = stage_row(st, p.sg_gu, L.g);
      const uint8_t* r1 = stage_row(st, p.sg_gu, L.g + 8);
      float gs = 0.f, us = 0.f;
      if (ok)
#pragma unroll 1
        for (int seg = hf ? nsg_lo : 0; seg < (hf ? nsg : nsg_lo); seg++) seg_dot<SG>(r0, r1, seg, xt, L, bf, gs, us);
      gs += __shfl_xor_sync(0xffffffffu, gs, 1);
      us += __shfl_xor_sync(0xffffffffu, us, 1);
      gs += __shfl_xor_sync(0xffffffffu, gs, 2);
      us += __shfl_xor_sync(0xffffffffu, us, 2);
      pair_sum(gs, us, it);  // both warps are done with the stage past this point
      if (!hf) {
        // lane (g, 0) holds gate row g and its up row (rows g and g + 8 of
        // the unit): the reference's SwiGLU, gguf_run.c:206
        if (L.t == 0 && ok) p.s.hbuf[(size_t)t * fe + 8 * (u0 + i) + L.g] = (gs / (1.0f + expf(-gs))) * us;
        __syncwarp();
        if (p.trace && lane == 0 && i < kTrItems) atomicMax(&ctl->it_done[i], now_ns());
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
    }
  }
  if (nDI > 0)
    g_to_d(true);
  else if (active)
    g_to_d(false);  // no down tiles here: publish the units only

  // ---- down tiles: the CTA's tile u to pair u mod NP; the last tile of an
  // item to finish releases its stage ------------------------------------------
  const int nDT = nDI > 0 ? nD : 0;
  if (q < NP) {
#pragma unroll 1
    for (int u = q, it = 0; u < nDT; u += NP, it++) {
      const int i = nG + u / P, tt = u - (u / P) * P;
      const int slot = i % S;
      const int nt = min(P, nD - (i - nG) * P);
      const bool ok = item_wait(full, ctl, p.s.err, i, S);
      if (p.trace && lane == 0 && !hf && i < kTrItems) atomicMin(&ctl->it_land[i], now_ns());
      const uint8_t* base = stages + (size_t)slot * p.stage_bytes + (size_t)tt * p.dslot_bytes;
      const uint8_t* r0 = stage_row(base, p.sg_d, L.g);
      const uint8_t* r1 = stage_row(base, p.sg_d, L.g + 8);
      float y0 = 0.f, y1 = 0.f;
      if (ok)
#pragma unroll 1
        for (int seg = hf ? nsd_lo : 0; seg < (hf ? nsd : nsd_lo); seg++) seg_dot<SD>(r0, r1, seg, ht, L, bf, y0, y1);
      y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
      y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
      y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
      y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
      pair_sum(y0, y1, it);
      if (!hf) {
        const int tile = i0 + u;
        if (L.t == 0 && ok) {
          p.s.ybuf[(size_t)t * d + 16 * tile + L.g] = y0;
          p.s.ybuf[(size_t)t * d + 16 * tile + L.g + 8] = y1;
        }
        __syncwarp();
        if (p.trace && lane == 0 && i < kTrItems) atomicMax(&ctl->it_done[i], now_ns());
        if (lane == 0 && atomicAdd(&ucnt[slot * kMaxDTiles], 1) == nt - 1) {
          ucnt[slot * kMaxDTiles] = 0;
          mbar_arrive(&empty[slot]);
        }
      }
    }
  }
  // count this CTA's tiles, one warp per tile, all at once (the down rows
  // stored above are made visible first); the last of the k experts to
  // finish a tile combines it
  __threadfence();
  named_bar(1, NC);
  for (int jj = warp; jj < nD; jj += W) count_tile(i0 + jj);
  if (threadIdx.x == 0) trace(p, kTrDDone);
  if (p.trace && threadIdx.x < kTrItems) {
    const unsigned long long ld = ctl->it_land[threadIdx.x];
    p.trace[blockIdx.x * kTraceSlots + 32 + threadIdx.x] = ld == ~0ull ? 0ull : ld;
    p.trace[blockIdx.x * kTraceSlots + 48 + threadIdx.x] = ctl->it_done[threadIdx.x];
  }

  // ---- launch exit: the last CTA out resets the per-launch words -------------
  named_bar(1, NC);
  if (threadIdx.x == 0) {
    // host-memory outputs (the host entry's residual rows and selection) are
    // visible system-wide before this CTA counts out, so the word the last
    // CTA writes tells the host that every output is in place
    if (p.err_out) __threadfence_system();
    if (atom_add_acq_rel_gpu(&sy->exit_cnt.v, 1u) == (unsigned)G - 1u) {
      if (p.err_out) {
        reinterpret_cast<volatile int*>(p.err_out)[0] = *reinterpret_cast<volatile int*>(p.s.err);
        __threadfence_system();
        reinterpret_cast<volatile int*>(p.err_out)[1] = 1;  // done
      }
      sy->router_arrive.v = 0u;
      for (int tt = 0; tt < k; tt++) sy->group[tt].v = 0u;
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
  const VecTab xt = {smem + p.off_xtab, reinterpret_cast<float*>(smem + p.off_xmeta), smem + p.off_xrtab,
                     reinterpret_cast<float*>(smem + p.off_xrmeta)};
  uint8_t* stages = smem + p.off_stage;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = kConsumerWarps;
  constexpr int NC = W * 32;
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
  // the weight rows do not depend on the previous kernel: start them toward
  // L2 while it finishes
  if (p.prefetch_bytes && threadIdx.x == 0 && nU > 0)
    prefetch_l2(p.W + (size_t)(16 * u0) * p.sg.rb,
                (uint32_t)min((uint64_t)(16 * nU) * p.sg.rb, (uint64_t)p.prefetch_bytes));
  pdl_launch_dependents();
  pdl_wait();
  __syncthreads();

  if (warp >= W) {
    produce_ring(full, empty, stages, p.stage_bytes, S, nU, ctl, p.err, [&](int v, int slot, uint8_t* st) {
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], 16u * p.sg.rb);
      __syncwarp();
      const uint8_t* src = p.W + (size_t)(16 * (u0 + v)) * p.sg.rb;
      issue_tile_bulk(st, &full[slot], src, src + 8 * (size_t)p.sg.rb, p.sg, lane);
    });
    return;
  }
  // x table (consumers only; the producer already streams weights), built
  // in place over the staged x
  {
    float* xs = reinterpret_cast<float*>(xt.tab);
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
    build_tables<SF>(xs, xt, nseg, warp, W, lane);
    named_bar(1, NC);
  }
  const LaneCtx L = lane_ctx();
  BFrag bf;
  bf.reset();
  for (int v = 0; v < nU; v++) {
    const int slot = v % S;
    const bool ok = warp_wait(&full[slot], (uint32_t)(v / S) & 1u, ctl, p.err);
    float val = 0.f;
    const bool last = consume_unit<SF>(stages + (size_t)slot * p.stage_bytes, p.sg, v, ok ? nseg : 0, W, warp, xt,
                                       part + slot * p.part_stride, &ucnt[slot], L, &val, bf);
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

bool fast_format(uint32_t type) { return type == T_Q8_0 || type == T_Q4_K || type == T_Q6_K || type == T_Q5_0; }

// Rows per copy group.  A group is G consecutive rows copied densely by one
// bulk copy (the copy engine spends about the same time on a copy of 1 KB as
// of 8 KB, so groups keep the copies few and large); groups are padded to
// start 16 B apart modulo 128 B.  G is at most 8 and at least the rows that
// make a multiple of 16 bytes; within that, the rows a warp reads together
// lie rb apart inside a group, and a bank model of each segment kernel's
// shared loads gives: Q6_K conflict-free for G <= 128 / gcd(rb, 128); Q8_0
// and Q5_0 (17 and 11 4-byte loads per segment, cheap next to a copy) at
// most two-way for twice that; Q4_K's 16-byte loads two wavefronts per
// quarter warp instead of one at G = 8.
static uint32_t copy_group_rows(uint32_t type, uint32_t rb) {
  const uint32_t gmin = 16u / gcd_u(rb, 16u);
  const uint32_t spread = 128u / gcd_u(rb, 128u);
  uint32_t g = type == T_Q4_K ? 8u : type == T_Q6_K ? spread : 2u * spread;
  if (g > 8u) g = 8u;
  return g < gmin ? gmin : g;
}

int stage_geom(uint32_t type, int K, StageGeom* sg) {
  if (!fast_format(type) || K <= 0 || K % kSegElems) return VIREO_ERR_UNSUPPORTED;
  int be, bb;
  if (type_block(type, &be, &bb)) return VIREO_ERR_UNSUPPORTED;
  const uint32_t rb = (uint32_t)(K / be) * (uint32_t)bb;
  const uint32_t G = copy_group_rows(type, rb);
  if (G > 8) return VIREO_ERR_UNSUPPORTED;
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
static const void* moe_kernel_ptr(bool routed) {
  return routed ? reinterpret_cast<const void*>(&moe_routed_kernel<SG, SD>)
                : reinterpret_cast<const void*>(&moe_decode_kernel<SG, SD>);
}

template <class SG>
static const void* moe_kernel_for(uint32_t dtype, bool routed) {
  if (dtype == T_Q8_0) return moe_kernel_ptr<SG, SegQ8>(routed);
  if (dtype == T_Q4_K) return moe_kernel_ptr<SG, SegQ4K>(routed);
  if (dtype == T_Q6_K) return moe_kernel_ptr<SG, SegQ6K>(routed);
  if (dtype == T_Q5_0) return moe_kernel_ptr<SG, SegQ5>(routed);
  return nullptr;
}

const void* moe_decode_kernel_for(uint32_t gtype, uint32_t dtype, bool routed) {
  if (gtype == T_Q8_0) return moe_kernel_for<SegQ8>(dtype, routed);
  if (gtype == T_Q4_K) return moe_kernel_for<SegQ4K>(dtype, routed);
  if (gtype == T_Q6_K) return moe_kernel_for<SegQ6K>(dtype, routed);
  if (gtype == T_Q5_0) return moe_kernel_for<SegQ5>(dtype, routed);
  return nullptr;
}

// Shared-memory layout for the MoE kernel; picks the deepest stage ring that
// fits.  Returns the dynamic shared-memory bytes (0 if nothing fits).
uint32_t moe_decode_layout(MoeDecodeParams* p, uint32_t smem_limit, int grid) {
  // a stage holds one gate/up unit or the whole number of down tiles nearest
  // to the same bytes (the stage grows to fit them)
  const uint32_t gstage = up_to(2u * p->sg_gu.hstride, 128u);  // one gate/up unit
  const uint32_t dslot = up_to(2u * p->sg_d.hstride, 16u);     // one down tile
  const uint32_t dt = std::min<uint32_t>(std::max<uint32_t>((gstage + dslot / 2) / dslot, 1u), (uint32_t)kMaxDTiles);
  const uint32_t stage = up_to(std::max(gstage, dt * dslot), 128u);
  p->stage_bytes = stage;
  p->dslot_bytes = dslot;
  p->dtiles = (int)dt;
  const int nsg = p->d / kSegElems, nsd = p->fe / kSegElems;
  int np = 64;  // the routing keys: ne rounded up to a power of two
  while (np < p->ne) np <<= 1;
  (void)nsg;
  (void)nsd;
  uint32_t off = 2u * kMaxStages * 8u;  // full/empty barriers
  p->off_ctl = off;
  off = up_to(off + (uint32_t)sizeof(Ctl), 16);
  p->off_etab = off;
  off = up_to(off + (uint32_t)(3 * p->ne * sizeof(void*)), 16);
  p->off_ucnt = off;
  off = up_to(off + (uint32_t)(kMaxStages * kMaxDTiles * 4), 16);
  p->off_xtab = off;  // x tables (the staged x before that)
  off = up_to(off + (uint32_t)(nsg * kSegTabBytes), 16);
  p->off_xmeta = off;
  off = up_to(off + (uint32_t)(nsg * kMeta * 4), 16);
  p->off_xrtab = off;
  off = up_to(off + (uint32_t)(nsg * kResTabBytes), 16);
  p->off_xrmeta = off;
  off = up_to(off + (uint32_t)(nsg * kMeta * 4), 16);
  p->off_htab = off;  // one expert's h tables; the routing keys before that
  off = up_to(off + (uint32_t)std::max(nsd * kSegTabBytes, 8 * std::max(64, np)), 16);
  p->off_hmeta = off;
  off = up_to(off + (uint32_t)(nsd * kMeta * 4), 16);
  p->off_hrtab = off;
  off = up_to(off + (uint32_t)(nsd * kResTabBytes), 16);
  p->off_hrmeta = off;
  off = up_to(off + (uint32_t)(nsd * kMeta * 4), 16);
  p->off_xs = off;  // residual rows of a CTA's tiles: at most d / 16 / floor(grid / k) + 1 tiles
  off = up_to(off + (uint32_t)(64 * (p->d / 16 / std::max(1, grid / std::max(1, p->k)) + 1)), 16);
  p->off_part = off;  // warp pairs' row-sum exchange: [pairs][2 parities][16] floats
  off = up_to(off + (uint32_t)(kConsumerWarps / 2 * 32 * 4), 16);
  for (int S = kMaxStages; S >= 2; S--) {
    const uint32_t st = up_to(off, 128);
    const uint32_t total = st + (uint32_t)S * stage;
    if (total <= smem_limit) {
      p->nstages = S;
      p->off_stage = st;
      return total;
    }
  }
  return 0;
}

static size_t up256s(size_t v) { return (v + 255) & ~(size_t)255; }

size_t moe_scratch_bytes(int d, int fe, int ne, int k) {
  size_t off = 0;
  off = up256s(off + sizeof(MoeSync));
  off = up256s(off + sizeof(int));                                       // status
  off = up256s(off + (size_t)(d / 16) * kTileCntStride * 4);              // tile counters
  off = up256s(off + 4 * (size_t)ne);                                     // router logits
  off = up256s(off + 4 * (size_t)k * fe);                                 // h
  off = up256s(off + 4 * (size_t)k * d);                                  // down outputs
  return off;
}

void moe_scratch_carve(uint8_t* base, int d, int fe, int ne, int k, int* err, MoeScratch* s) {
  size_t off = 0;
  s->sync = (MoeSync*)(base + off);
  off = up256s(off + sizeof(MoeSync));
  s->err = err ? err : (int*)(base + off);
  off = up256s(off + sizeof(int));
  s->tile_cnt = (unsigned int*)(base + off);
  off = up256s(off + (size_t)(d / 16) * kTileCntStride * 4);
  s->logit_part = (float*)(base + off);
  off = up256s(off + 4 * (size_t)ne);
  s->hbuf = (float*)(base + off);
  off = up256s(off + 4 * (size_t)k * fe);
  s->ybuf = (float*)(base + off);
}

const void* gemv_kernel_for(uint32_t type) {
  if (type == T_Q8_0) return reinterpret_cast<const void*>(&gemv_kernel<SegQ8>);
  if (type == T_Q4_K) return reinterpret_cast<const void*>(&gemv_kernel<SegQ4K>);
  if (type == T_Q6_K) return reinterpret_cast<const void*>(&gemv_kernel<SegQ6K>);
  if (type == T_Q5_0) return reinterpret_cast<const void*>(&gemv_kernel<SegQ5>);
  return nullptr;
}

// Shared-memory layout for gemv_kernel: the deepest ring that fits, and no
// deeper than the max_units units a CTA streams (at least 2 stages).
uint32_t gemv_layout(GemvParams* p, uint32_t smem_limit, int max_units) {
  const int W = kConsumerWarps, nseg = p->n / kSegElems;
  const uint32_t stage = up_to(2u * p->sg.hstride, 128u);
  p->stage_bytes = stage;
  p->part_stride = (uint32_t)std::max(W, nseg) * 16u;
  for (int S = std::max(2, std::min(kMaxStages, max_units)); S >= 2; S--) {
    uint32_t off = 2u * kMaxStages * 8u;
    p->off_ctl = off;
    off = up_to(off + (uint32_t)sizeof(Ctl), 16);
    p->off_part = off;
    off = up_to(off + (uint32_t)S * p->part_stride * 4u, 16);
    p->off_ucnt = off;
    off = up_to(off + (uint32_t)(S * 4), 16);
    p->off_xtab = off;  // x tables (the staged x before that)
    off = up_to(off + (uint32_t)(nseg * kSegTabBytes), 16);
    p->off_xmeta = off;
    off = up_to(off + (uint32_t)(nseg * kMeta * 4), 16);
    p->off_xrtab = off;
    off = up_to(off + (uint32_t)(nseg * kResTabBytes), 16);
    p->off_xrmeta = off;
    off = up_to(off + (uint32_t)(nseg * kMeta * 4), 128);
    p->off_stage = off;
    off += (uint32_t)S * stage;
    if (off <= smem_limit) {
      p->nstages = S;
      return off;
    }
  }
  return 0;
}

}  // namespace vireo
