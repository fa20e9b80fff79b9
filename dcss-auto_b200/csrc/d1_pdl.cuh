// Programmatic dependent launch (sm_90 and later) for chains of kernels on one
// stream, such as a PPO minibatch: a kernel launched with the attribute of
// pdl_config() may be launched while the previous kernel of its stream is still
// finishing, so that its launch and prologue overlap that kernel's end.
// pdl_wait() then blocks until the previous kernel has completed and its memory
// writes are visible. Every kernel launched this way calls it in every block
// before its first global-memory read or write (only shared memory, barriers,
// tensor memory and parameters are touched before it). For a kernel launched
// without the attribute it returns at once.
#pragma once
#include <cuda_runtime.h>

namespace d1 {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// A launch configuration whose single attribute allows the programmatic
// overlap; `attr` must outlive the launch call.
inline cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                     cudaLaunchAttribute *attr) {
    attr->id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr->val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

}  // namespace d1
