// Programmatic dependent launch (PDL) for every kernel of the hot path.
//
// Each kernel is launched with the programmatic-stream-serialization
// attribute, lets its dependents launch early (griddepcontrol.launch_dependents)
// and waits for its predecessor (griddepcontrol.wait) after its prologue and
// before touching memory the predecessor may read or write.  The dependent
// grid only launches once every CTA of this grid has started, so CTAs of two
// kernels never starve each other, and griddepcontrol.wait blocks until the
// predecessor grid has completed and its writes are visible: the stream order
// of the data is unchanged, only launch latency and prologues overlap.
// CUDA-graph capture keeps these launches as programmatic edges.  SH_PDL=0
// launches without the attribute (griddepcontrol.wait is then a no-op).
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>
#include <utility>

namespace shk {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("SH_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace shk
