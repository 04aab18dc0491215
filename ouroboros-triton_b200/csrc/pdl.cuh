// Launch with programmatic stream serialization (programmatic dependent launch):
// the kernel's CTAs may be scheduled before the previous kernel on the stream has
// completed, once that kernel's CTAs have all executed griddepcontrol.launch_dependents
// (or exited). Every kernel launched this way calls griddep_wait() before it touches
// memory that earlier work on the stream writes or reads; after that call the previous
// kernels are complete and their writes visible, exactly as with a plain launch.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace ouro {

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace ouro
