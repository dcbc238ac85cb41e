// Host-side launch with programmatic stream serialization for the batched
// (prefill) and expert-parallel kernels.  The kernel may be scheduled while
// the previous kernel on the stream is still running; every kernel launched
// this way begins with pdl_wait() (griddepcontrol.wait), which returns once
// the preceding kernel has completed and its memory is visible, so stream
// order is kept for every read and write and only the launch latency
// overlaps the previous kernel's tail.
#pragma once

#include <cuda_runtime.h>

#include <utility>

#include "vireo_internal.h"

namespace vireo {

template <typename... KArgs, typename... Args>
inline int pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
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

}  // namespace vireo
