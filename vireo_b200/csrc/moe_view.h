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

}  // namespace vireo
