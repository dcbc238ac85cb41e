// Batch-1 MoE FFN decode: one kernel launch per token.
//
// Replaces, for one token, the reference's moe_ffn (vireo src/gguf_run.c:
// 185-214): router matvec (:187), softmax (:181-182, :188), greedy top-k
// with ties to the lowest expert id (:190-191), optional renormalisation
// (:192), per expert gate/up matvec + SwiGLU + down matvec (:198-208), the
// weighted combine in rank order (:209) and the residual add (:213).
//
// One CTA per SM, every CTA resident (each cross-CTA wait is bounded).
//   R  router logits, one warp per expert row (512-value chunks summed in
//      order) -> grid arrival counter -> in every CTA the producer warp
//      reads the ne logits, takes the softmax and selects the top-k
//      (k rounds of a warp arg-max) while the consumer warps build the
//      activation tables of x.
//   The CTAs are then split into k groups, group t serving the expert of
//   rank t.  A CTA of group t streams, through one ring of shared-memory
//   stages, its share of that expert's gate/up units (8 gate + 8 up rows)
//   and then its share of the expert's down tiles (16 rows; several per
//   stage), so the down rows arrive while gate/up is still computed.
//   G  unit i to consumer warp group i mod (W / g) (g = 2 warps for Q8_0
//      gate/up rows, each running half of the segments and adding the
//      halves; g = 1 otherwise), which writes h = silu(g) * u for its 8 rows
//      to scratch; the group counts finished units.
//   D  once the group's units are all counted, the CTA stages the expert's h
//      and builds its activation tables; down tile u to warp group
//      u mod (W / g), which writes its 16 outputs to scratch; then every
//      tile is counted and the last of the k groups to finish a tile
//      combines the k experts' rows in rank order and adds them into the
//      residual.
#pragma once
#include <stdint.h>

#include "engine.cuh"

namespace vireo {

constexpr int kConsumerWarps = 15;
constexpr int kProducerWarps = 1;  // issues the bulk weight copies
constexpr int kDecodeThreads = 32 * (kConsumerWarps + kProducerWarps);
constexpr int kMaxDTiles = 4;      // down tiles per ring stage
constexpr int kRouterChunk = 512;
constexpr int kMaxTopK = 64;
constexpr int kMaxExperts = 256;
constexpr int kMaxHValues = 8192;  // n_used * ffn_exp
constexpr int kTileCntStride = 32;  // words between two tiles' counters (one 128-byte line each)

// Per-launch synchronisation words in device scratch.  All start at zero;
// the last CTA to leave a launch puts them back to zero.
// Each word sits on its own 256-byte line: words that many CTAs update must
// not share an L2 line, or their atomics queue behind one another.
struct alignas(256) SyncWord {
  unsigned int v;
  unsigned int pad[63];
};
struct MoeSync {
  SyncWord router_arrive;    // CTAs done with their router partials
  SyncWord exit_cnt;         // CTAs done with the launch
  SyncWord group[kMaxTopK];  // gate/up units finished per expert slot
};

// Device scratch of one layer handle (or of the fixed no-allocation array).
struct MoeScratch {
  float* logit_part;        // [ne] router logits
  float* hbuf;              // [k][fe] h rows of the selected experts
  float* ybuf;              // [k][d] down outputs of the selected experts
  unsigned int* tile_cnt;   // [d/16][kTileCntStride]: expert rows finished per 16-row tile; back to 0 by the combiner
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
  uint32_t stage_bytes;  // ring stage: one gate/up unit or dtiles down tiles
  int nstages;
  uint32_t dslot_bytes;  // one down tile inside a stage
  int dtiles;            // down tiles per stage
  // shared-memory offsets (bytes)
  uint32_t off_ctl, off_etab, off_ucnt, off_part, off_xtab, off_xmeta, off_xrtab, off_xrmeta, off_htab, off_hmeta,
      off_hrtab, off_hrmeta, off_xs, off_stage;
  unsigned long long* trace;  // optional: kTraceSlots %globaltimer stamps per CTA
  // optional (decoder): hb is not given; every CTA forms x + res_y (the
  // residual add before the FFN) and its RMSNorm with norm_w as the hidden
  // vector, and x + res_y is the residual the output is added to
  const float* res_y;
  const float* norm_w;
  float norm_eps;
  // optional (shared expert, routed launches): the weight of slot 0 is
  // sigmoid(sh_gate . hb), formed by every CTA, instead of the route's
  const float* sh_gate;
  int* err_out;               // optional, mapped host memory: the last CTA out writes the status word to
                              // [0], then 1 to [1]
};

// Scratch bytes of a layer and the pointers into a block of that size (256-
// byte aligned); the sync words and the tile counters must start at zero.
size_t moe_scratch_bytes(int d, int fe, int ne, int k);
void moe_scratch_carve(uint8_t* base, int d, int fe, int ne, int k, int* err, MoeScratch* s);

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
  kTrProdFirst, kTrProdFirstD, kTrProdLast, kTrProdDrained, kTrPdl,
  kTrDbg = 64, kTraceSlots = 72
};

struct GemvParams {
  const uint8_t* W;  // [d][row bytes] raw GGUF rows
  const float* x;    // [n]
  float* y;          // [d]
  int n, d;
  StageGeom sg;
  uint32_t stage_bytes;
  int nstages;
  uint32_t off_part, off_ucnt, off_ctl, off_xtab, off_xmeta, off_xrtab, off_xrmeta, off_stage;
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
