// Host-side launch helper for programmatic dependent launch (PDL).
//
// A kernel launched with launch_pdl may begin (prologue, TMEM allocation,
// prefetch of data no earlier kernel writes) while the previous kernel in the
// stream is still running. Every such kernel calls pdl_wait() (common.cuh)
// before it reads anything an earlier kernel produced or writes anything an
// earlier kernel reads, and pdl_trigger() only after that wait, so at most the
// immediately preceding kernel is still running during its pre-wait prologue.
// ISB_PDL=0 in the environment launches everything with plain stream order.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <utility>

namespace isb {

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("ISB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace isb
