// launch.cuh -- kernel launches with an optional programmatic dependency on
// the previous work of the stream (CUDA programmatic dependent launch): the
// kernel may start while that work is still running, and must call
// griddep_wait() (ptx.cuh) before it touches anything that work writes or
// reads, and before it exits.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace tir {

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace tir
