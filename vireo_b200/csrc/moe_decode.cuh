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
#pragma once
#include <stdint.h>

#include "engine.cuh"

namespace vireo {

constexpr int kConsumerWarps = 8;
constexpr int kDecodeThreads = 32 * (kConsumerWarps + 1);
constexpr int kRouterChunk = 512;
constexpr int kMaxTopK = 64;

struct MoeScratch {
  float* logit_part;       // [d/512][ne]
  float* hbuf;             // [k][fe]
  float* ybuf;             // [k][d]
  unsigned int* tile_cnt;  // [d/16]
  GridSync* gsync;
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
  uint32_t stage_bytes;
  int nstages;
  // shared-memory offsets (bytes)
  uint32_t off_part, off_ucnt, off_ctl, off_xtab, off_xsx, off_htab, off_hsx, off_stage;
  uint32_t htab_bytes;  // per expert table bytes
};

struct GemvParams {
  const uint8_t* W;  // [d][row bytes] raw GGUF rows
  const float* x;    // [n]
  float* y;          // [d]
  int n, d;
  StageGeom sg;
  uint32_t stage_bytes;
  int nstages;
  uint32_t off_part, off_ucnt, off_ctl, off_xtab, off_xsx, off_stage;
  int* err;
};

}  // namespace vireo
