// What the expert-parallel path (ep.cu) reads of a gguf_moe layer handle
// (defined in api.cu).
#pragma once
#include <cuda_runtime.h>

#include "gguf_moe.h"
#include "vireo_internal.h"

namespace vireo {

struct MoeView {
  const gguf_moe_desc* desc;
  const uint8_t* const* exp_tab;
  PrefillScratch* pre;
  int* err;
  int num_sms;
  cudaStream_t stream;
};
int moe_view(gguf_moe* m, MoeView* v);

// One decode launch with the residual add and the FFN norm folded in: x +=
// y, then x += MoE(rmsnorm(x) * w) (the decoder's gguf_run.c:237-239).
int moe_ffn_norm(gguf_moe* m, float* x, const float* y, const float* w, float eps, cudaStream_t s);

}  // namespace vireo
