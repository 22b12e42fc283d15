// qw6_pdl.cuh -- programmatic dependent launch for chains of kernels on one
// stream (also inside CUDA graphs): a kernel launched with launch_pdl may be
// scheduled while its predecessor still runs, and must call pdl_wait()
// before it touches anything the predecessor writes (pdl_wait returns at
// once when the kernel was launched normally).  Such a kernel must not take
// data that an earlier kernel writes through `const T* __restrict__`: the
// compiler may then treat it as read-only for the kernel's whole life, read
// it through the non-coherent path and move the loads above the wait (on the
// B200 this returned stale rows); weights written once at upload may be.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace qw6 {

__device__ __forceinline__ void pdl_grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
#ifdef QW6_PDL_OFF  // diagnostic builds: plain stream order
    at[0].val.programmaticStreamSerializationAllowed = 0;
#else
    at[0].val.programmaticStreamSerializationAllowed = 1;
#endif
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace qw6
