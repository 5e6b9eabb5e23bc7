// launch.cuh -- kernel launches with an optional programmatic dependency on
// the previous work of the stream (CUDA programmatic dependent launch): the
// kernel may start while that work is still running, and must call
// griddep_wait() (ptx.cuh) before it touches anything that work writes or
// reads, and before it exits.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace tir {

// As launch_kernel, in thread-block clusters of `cluster` CTAs (1 x 1 x 1:
// no cluster).
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                  bool pdl, dim3 cluster, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster.x * cluster.y * cluster.z > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster.x;
        attr[n].val.clusterDim.y = cluster.y;
        attr[n].val.clusterDim.z = cluster.z;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          bool pdl, Args&&... args) {
    return launch_kernel_cluster(kernel, grid, block, smem, stream, pdl, dim3(1, 1, 1), std::forward<Args>(args)...);
}

}  // namespace tir
