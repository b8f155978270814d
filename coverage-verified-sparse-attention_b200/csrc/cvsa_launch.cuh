// Kernel launch helper: optional programmatic dependent launch (PDL), so a
// kernel's CTAs are scheduled while its predecessor drains; the kernel itself
// calls griddepcontrol.wait before touching the predecessor's outputs.
#pragma once

#include <cuda_runtime.h>

namespace cvsa {

template <typename Kernel, typename... Args>
cudaError_t launch_k(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace cvsa
