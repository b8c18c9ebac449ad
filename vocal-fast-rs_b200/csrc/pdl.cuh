// Programmatic dependent launch between the kernels of one call.
//
// A kernel launched by launch_pdl may be scheduled while the kernel before
// it on the stream is still running (once every CTA of that kernel has
// called launch_dependents(), or has exited), so its prologue overlaps the
// predecessor's tail.  It must call grid_dependency_wait() before it reads
// anything the predecessor writes, or writes anything the predecessor
// reads; the wait returns once the predecessor has completed and its memory
// operations are visible.  In a kernel launched without the attribute both
// instructions return at once.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace vfr {

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
    cudaLaunchConfig_t cfg{};
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

}  // namespace vfr
