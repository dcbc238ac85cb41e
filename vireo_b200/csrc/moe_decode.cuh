// Batch-1 MoE FFN decode: one persistent cooperative kernel per token.
//
// Replaces, for one token, the reference's moe_ffn (vireo src/gguf_run.c:
// 185-214): router matvec (:187), softmax (:181-182, :188), greedy top-k
// with ties to the lowest expert id (:190-191), optional renormalisation
// (:192), per expert gate/up matvec + SwiGLU + down matvec (:198-208), the
// weighted combine in rank order (:209) and the residual add (:213).
//
// Phases (one CTA per SM, all co-resident):
//   R  router partial dot products, 512-value K chunks, one warp per task
//      -> grid barrier ->
//      every CTA sums the partials in chunk order, softmax, top-k, renorm
//   G  units (expert slot t, 8 rows): 8 gate rows + 8 up rows per MMA tile,
//      epilogue h = silu(g) * u into scratch
//      -> grid barrier (consumers only; the producer keeps streaming the
//         down rows, which do not depend on h) ->
//   D  units (expert slot t, 16 rows of the down matrix); epilogue writes the
//      expert's rows and the last of the k experts to finish a 16-row tile
//      combines them in rank order into the residual.
// The weight stages form two rings over one shared-memory area: gate/up
// units in stages sized for them, down units in (usually smaller) slots of
// their own, so that more down units are in flight during gate/up.
#pragma once
#include <stdint.h>

#include "engine.cuh"

namespace vireo {

constexpr int kConsumerWarps = 12;
constexpr int kProducerWarps = 4;  // issue the 16-byte cp.async weight copies
constexpr int kProducerThreads = 32 * kProducerWarps;
constexpr int kDecodeThreads = 32 * (kConsumerWarps + kProducerWarps);
constexpr int kRouterChunk = 512;
constexpr int kMaxTopK = 64;
constexpr int kMaxHValues = 8192;  // n_used * ffn_exp: h scratch and the down tables in shared memory

// Per-launch synchronisation words in device scratch.  All start at zero;
// the last CTA to leave a launch puts them back to zero.
// Each word sits on its own 256-byte line: words that many CTAs update must
// not share an L2 line, or their atomics queue behind one another.
struct alignas(256) SyncWord {
  unsigned int v;
  unsigned int pad[63];
};
struct MoeSync {
  SyncWord router_arrive;  // CTAs done with their router partials
  SyncWord g_done;         // gate/up units finished (added once per CTA)
  SyncWord exit_cnt;       // CTAs done with the launch
};

struct MoeScratch {
  float* logit_part;  // [d/512][ne]
  float* hbuf;        // [k][fe]
  MoeSync* sync;
  int* err;
};

struct MoeDecodeParams {
  int d, fe, ne, k, renorm;
  const float* router;               // [ne][d] fp32
  const uint8_t* const* exp_tab;     // [ne][3] device pointers: gate, up, down
  const float* hb;                   // [d] normalised hidden
  float* x;                          // [d] residual, in/out
  int32_t* ids_out;                  // [k] or null
  float* wts_out;                    // [k] or null
  MoeScratch s;
  StageGeom sg_gu, sg_d;
  uint32_t stage_bytes;  // gate/up ring: nstages stages of stage_bytes
  int nstages;
  uint32_t dslot_bytes;  // down ring: nstages_d slots of dslot_bytes over the same memory
  int nstages_d;
  // shared-memory offsets (bytes)
  uint32_t off_part, off_part_d, off_ucnt, off_ytile, off_ctl, off_xtab, off_xsx, off_htab, off_hsx, off_stg,
      off_stage;
  uint32_t htab_bytes;  // per expert table bytes
  uint32_t hsx_count;   // activation metadata floats per expert table
  uint32_t part_stride; // floats of segment partials per stage
  unsigned long long* trace;  // optional: kTraceSlots %globaltimer stamps per CTA
};

// A route given by the caller (routed launches, no router phase): rank-order
// expert ids (-1 = unused slot), gate weights as used in the combine, and the
// device addresses of each selected expert's gate, up and down slices.
// Passed by value as a kernel parameter (2 KB).
struct MoeRoute {
  int ids[kMaxTopK];
  float wts[kMaxTopK];
  const uint8_t* ptr[kMaxTopK][3];
};

// phase trace slots (per CTA): consumer thread 0 and producer thread 0
enum TraceSlot {
  kTrStart = 0, kTrRouterDone, kTrPartials, kTrRouted, kTrGDone, kTrGAll, kTrHtab, kTrDDone,
  kTrProdFirst, kTrProdFirstD, kTrProdLast, kTrProdDrained,
  kTrUnitBase = 16,  // per-unit stamps for the first kTrUnits units: ready, done
  kTrUnits = 24, kTrDbg = 64, kTraceSlots = 72
};

struct GemvParams {
  const uint8_t* W;  // [d][row bytes] raw GGUF rows
  const float* x;    // [n]
  float* y;          // [d]
  int n, d;
  StageGeom sg;
  uint32_t stage_bytes;
  int nstages;
  uint32_t off_part, off_ucnt, off_ctl, off_xtab, off_xsx, off_stg, off_stage;
  uint32_t part_stride;
  int* err;
  // optional, zero by default: y = W . rmsnorm(x, norm_w, eps) (the norm
  // computed by every CTA from x), and an L2 prefetch of up to
  // prefetch_bytes of the CTA's weight rows issued before the kernel waits
  // on its predecessor (weights are not written by the kernels of a step)
  const float* norm_w;
  float eps;
  uint32_t prefetch_bytes;
};

}  // namespace vireo
