// Programmatic dependent launch (sm_90+) for the streaming kernels.
//
// A kernel launched with cudaLaunchAttributeProgrammaticStreamSerialization
// may be scheduled while the previous kernel of its stream is still running;
// pdl_enter() at its start waits (griddepcontrol.wait, a hardware wait, not a
// loop) until that kernel has completed and its memory is visible, before
// any global memory is touched, and then lets this kernel's own dependents be
// scheduled (griddepcontrol.launch_dependents).  Back-to-back steps then
// overlap one kernel's launch and ramp-up with the previous one's tail.  A
// kernel launched without the attribute passes both instructions at once.
#pragma once

#include <cuda_runtime.h>

namespace askb {

__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace askb
