// Kernel launches with the sm_100a launch attributes the engine uses.
//
// Programmatic dependent launch: while `t_pdl_launch` is set (the engine sets
// it around the launches of small passes), kernels are launched with
// programmatic stream serialisation, so a kernel's CTAs may start - and run
// their set-up (barrier init, TMEM allocation, descriptor prefetch) - while
// the previous kernel on the stream is finishing.  Every kernel of the engine
// calls pdl_launch_dependents() on entry and pdl_wait() before its first
// global-memory access; without the attribute both are no-ops.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace lama {

extern thread_local bool t_pdl_launch;

template <class... KArgs, class... Args>
int launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster,
                  Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    n++;
  }
  if (t_pdl_launch) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return (int)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace lama
