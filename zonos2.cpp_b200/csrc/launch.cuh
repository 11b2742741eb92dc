// launch.cuh — kernel launch with programmatic dependent launch (PDL).
//
// Every kernel of the decode step is launched with programmatic stream serialization:
// a kernel may start while its predecessor drains, runs only prologue work that reads
// no predecessor output (barrier init, TMA prefetch of static weights), then waits with
// griddepcontrol.wait before touching step data, and releases its own dependent with
// griddepcontrol.launch_dependents once it has passed that wait.
#pragma once

#include <cuda_runtime.h>
#include <utility>

namespace z2b {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" :::); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace z2b
