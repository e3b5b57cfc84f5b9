// Programmatic dependent launch (PDL) for the decode kernels.
//
// Every kernel of a decode step is launched with programmatic stream serialisation, so kernel N+1
// may start while kernel N still runs. The rule each kernel follows: before pdl_wait() it may only
// read constant data (weights) and compute indices; it writes nothing and reads no buffer that an
// earlier kernel produces. pdl_wait() returns once the previous kernel has completed and its
// memory is visible; by induction all earlier kernels have completed too. pdl_trigger() lets the
// next kernel begin its own constant-data prologue early.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace bst {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches `kernel` with programmatic stream serialisation allowed.
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
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(std::forward<Args>(args))...);
}

}  // namespace bst
