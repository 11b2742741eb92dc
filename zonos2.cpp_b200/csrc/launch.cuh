// launch.cuh — kernel launch for the decode step, with optional programmatic dependent
// launch (PDL).
//
// Every kernel is written for PDL: it runs only prologue work that reads no predecessor
// output (barrier init, bulk prefetch of static weights or cached KV) before
// griddepcontrol.wait, and releases its dependent with griddepcontrol.launch_dependents
// once past that wait. Without the launch attribute both instructions are no-ops. The
// attribute is off (kUsePdl): on the config-2 decode step, early-resident blocks of the
// next kernel cost more occupancy than the overlapped prologues saved (4.82 ms per step
// with PDL against 4.68 ms without, same box, back to back).
#pragma once

#include <cuda_runtime.h>
#include <utility>

namespace z2b {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" :::); }

constexpr bool kUsePdl = false;

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
    cfg.numAttrs = kUsePdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace z2b
