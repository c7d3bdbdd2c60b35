// Host-side launch helper for programmatic dependent launch (PDL).
//
// A kernel launched with launch_pdl may begin (prologue, TMEM allocation,
// prefetch) while earlier kernels in the stream are still running. Every such
// kernel calls pdl_trigger() (common.cuh) as it starts, so the next kernel can
// be scheduled once all of this kernel's CTAs are resident, and pdl_wait()
// before it reads anything an earlier kernel produced or writes anything an
// earlier kernel reads. pdl_wait() returns only after the previous kernel has
// completed, and that kernel completed only after its own wait returned, so the
// ordering is transitive. Several kernels of a chain can be in flight at once,
// and a dependent may also start before a plainly launched predecessor's writes
// are visible, so code before pdl_wait() reads only data no kernel ever writes
// (the weights).
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

// launch_pdl plus a thread-block-cluster shape.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                      dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster.x;
  attr[1].val.clusterDim.y = cluster.y;
  attr[1].val.clusterDim.z = cluster.z;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace isb
