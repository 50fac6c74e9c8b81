// Programmatic dependent launch (PDL) between the kernels of one forward.
//
// A kernel launched with programmatic stream serialization may start while
// the previous kernel on the stream is still running.  Every kernel of the
// decode chain therefore calls pdl_wait() before it touches memory written by
// earlier kernels (the quantized GEMV first issues its weight prefetch, which
// reads only immutable weights), and pdl_trigger() right after the wait, so
// the next kernel can begin its own prefetch.  Triggering only after the wait
// keeps at most two grids overlapping: the next grid is released once every
// CTA of the current one is running.  Without the launch attribute both
// instructions are no-ops.
#pragma once
#include <cuda_runtime.h>

#include <utility>

#include "common.h"

namespace wl {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// true while the calling host thread enqueues a forward (set by the runtime)
bool pdl_enabled();

template <class... KArgs, class... Args>
int launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  cfg.numAttrs = 0;
  if (pdl_enabled()) {
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cfg.attrs = at;
  WL_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
  return WL_OK;
}

}  // namespace wl
