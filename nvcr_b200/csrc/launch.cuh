// Programmatic dependent launch. A kernel launched with launch_overlapped may
// start (its prologue: barrier set-up, TMEM allocation, constant parameters,
// weight loads) while the kernels before it in the stream still run; every
// thread calls grid_dependency_wait() before it touches global memory those
// kernels write, or memory they read that it writes. launch_dependents() lets
// the next overlapped kernel start as this one's blocks finish.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace nvcr_sm100::kernels {

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... Params, typename... Args>
cudaError_t launch_overlapped(void (*kernel)(Params...), dim3 grid, dim3 block, std::size_t shared_bytes,
                              cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = shared_bytes;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

}  // namespace nvcr_sm100::kernels
